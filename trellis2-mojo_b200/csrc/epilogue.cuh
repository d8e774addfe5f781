// Conv epilogue shared by the tensor-core kernels: bias, SiLU, residual,
// conversion and the store of 16 consecutive output channels of one row.
// Args is any launch-argument struct with y, res (bytes), bias, co, flags.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/t2sc.h"

namespace t2sc {

constexpr int kEpiF32 = 3;  // f32 outputs (the split-TF32 mode), beside T2SC_DT_F16 / T2SC_DT_BF16

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (DT == T2SC_DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
}
template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if (DT == T2SC_DT_BF16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&v);
    return __bfloat1622float2(h);
  } else {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
  }
}

// v / (1 + exp(-v)); the exponent is clamped so the divisor stays in the
// range where the fast division is accurate (SiLU(v) for v < -80 is below
// 1e-33 either way).
__device__ __forceinline__ float silu(float v) { return __fdividef(v, 1.0f + __expf(fminf(-v, 80.0f))); }

// Epilogue for 16 consecutive output channels of one row.
template <int DT, class Args>
__device__ __forceinline__ void store16(const Args &a, int orow, int col, const float (&acc)[16]) {
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = acc[i] + __ldg(a.bias + col + i);
  if (a.flags & T2SC_SILU) {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = silu(v[i]);
  }
  if (DT == kEpiF32) {
    const int64_t off = ((int64_t)orow * a.co + col) * 4;
    if (a.flags & T2SC_RESIDUAL) {
      const float4 *rp = reinterpret_cast<const float4 *>(a.res + off);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        float4 r = __ldg(rp + q);
        v[4 * q] += r.x;
        v[4 * q + 1] += r.y;
        v[4 * q + 2] += r.z;
        v[4 * q + 3] += r.w;
      }
    }
    float4 *yp = reinterpret_cast<float4 *>(a.y + off);
#pragma unroll
    for (int q = 0; q < 4; q++) yp[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    return;
  }
  const int64_t off = ((int64_t)orow * a.co + col) * 2;
  if (a.flags & T2SC_RESIDUAL) {
    const uint4 *rp = reinterpret_cast<const uint4 *>(a.res + off);
    uint4 r0 = __ldg(rp), r1 = __ldg(rp + 1);
    uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float2 f = unpack2<DT>(rr[i]);
      v[2 * i] += f.x;
      v[2 * i + 1] += f.y;
    }
  }
  uint4 o0, o1;
  o0.x = pack2<DT>(v[0], v[1]);
  o0.y = pack2<DT>(v[2], v[3]);
  o0.z = pack2<DT>(v[4], v[5]);
  o0.w = pack2<DT>(v[6], v[7]);
  o1.x = pack2<DT>(v[8], v[9]);
  o1.y = pack2<DT>(v[10], v[11]);
  o1.z = pack2<DT>(v[12], v[13]);
  o1.w = pack2<DT>(v[14], v[15]);
  uint4 *yp = reinterpret_cast<uint4 *>(a.y + off);
  yp[0] = o0;
  yp[1] = o1;
}

}  // namespace t2sc
