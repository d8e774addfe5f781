// LayerNorm over the channel dim of sparse features, optionally followed by
// SiLU: the norm -> activation glue around the decoder convs
// (LayerNorm32.forward, trellis2_mojo/modules/nn.mojo:313-370; used as
// norm1/SiLU before conv1 and norm2/SiLU before conv2,
// models/sc_vaes/sparse_unet_vae.mojo:118,123). One warp per row: the row
// is read once into registers (C <= 1024), mean and population variance
// are warp-shuffle reductions in f32, inv_std = 1/sqrt(var + eps).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace t2sc {
namespace {

constexpr int kMaxPerLane = 32;  // C <= 1024

template <int DT>
__device__ __forceinline__ float ld(const void *p, int64_t i) {
  if (DT == T2SC_DT_F32) return static_cast<const float *>(p)[i];
  if (DT == T2SC_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}
template <int DT>
__device__ __forceinline__ void st(void *p, int64_t i, float v) {
  if (DT == T2SC_DT_F32)
    static_cast<float *>(p)[i] = v;
  else if (DT == T2SC_DT_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

template <int DT>
__global__ void __launch_bounds__(256) layernorm_kernel(const void *__restrict__ x, void *__restrict__ y, int64_t rows,
                                                        int c, const float *__restrict__ w,
                                                        const float *__restrict__ b, float eps, int silu) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = row * c;
  float v[kMaxPerLane];
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxPerLane; q++) {
    const int i = q * 32 + lane;
    v[q] = i < c ? ld<DT>(x, base + i) : 0.f;
    s += v[q];
  }
  const float mean = warp_sum(s) / (float)c;
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxPerLane; q++) {
    const int i = q * 32 + lane;
    const float d = i < c ? v[q] - mean : 0.f;
    ss += d * d;
  }
  const float inv_std = 1.0f / sqrtf(warp_sum(ss) / (float)c + eps);
#pragma unroll
  for (int q = 0; q < kMaxPerLane; q++) {
    const int i = q * 32 + lane;
    if (i < c) {
      float o = (v[q] - mean) * inv_std;
      if (w) o = o * w[i] + b[i];
      if (silu) o = o / (1.0f + expf(-o));
      st<DT>(y, base + i, o);
    }
  }
}

}  // namespace

int layernorm_device(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w, const float *b,
                     float eps, int flags, int dtype, std::string &err) {
  if (rows == 0) return T2SC_OK;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  const int silu = (flags & T2SC_SILU) ? 1 : 0;
  if (dtype == T2SC_DT_F32)
    layernorm_kernel<T2SC_DT_F32><<<blocks, 256, 0, ctx->stream>>>(x, y, rows, c, w, b, eps, silu);
  else if (dtype == T2SC_DT_BF16)
    layernorm_kernel<T2SC_DT_BF16><<<blocks, 256, 0, ctx->stream>>>(x, y, rows, c, w, b, eps, silu);
  else
    layernorm_kernel<T2SC_DT_F16><<<blocks, 256, 0, ctx->stream>>>(x, y, rows, c, w, b, eps, silu);
  T2SC_LAUNCHED(ctx, "layernorm");
  return T2SC_OK;
}

}  // namespace t2sc
