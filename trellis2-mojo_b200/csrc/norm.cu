// LayerNorm over the channel dim of sparse features, optionally followed by
// SiLU: the norm -> activation glue around the decoder convs
// (LayerNorm32.forward, trellis2_mojo/modules/nn.mojo:313-370; used as
// norm1/SiLU before conv1 and norm2/SiLU before conv2,
// models/sc_vaes/sparse_unet_vae.mojo:118,123). Each row is read once into
// registers (C <= 1024); mean and population variance are shuffle
// reductions in f32 over the row's lane group, inv_std = 1/sqrt(var + eps).
//
// The op moves 2·N·C·s bytes and does ~20 instructions per element, so it
// is HBM-bound only if enough bytes are in flight and the per-element math
// stays short:
//  - vector kernel (row bytes a multiple of 16, 16-byte aligned buffers): a
//    group of T lanes (a power of two, one to 32) owns a row, each lane V
//    16-byte chunks of it; every group handles R rows whose loads are all
//    issued before the first reduction (V·R = 8 chunks, 128 bytes in flight
//    per lane). For a fixed r the warp's groups read consecutive rows, so
//    each load instruction covers one contiguous span;
//  - scalar kernel (any C, any alignment): the same grouping over single
//    elements.
// SiLU is x / (1 + e^-x) with the fast exponential and division for f32
// outputs (the exponent clamped at 80 so the divisor stays finite; x < -80
// gives |silu| < 1e-33 either way) and 0.5 x (1 + tanh(x / 2)) with the
// hardware tanh for 16-bit outputs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace t2sc {
namespace {

__device__ __forceinline__ float silu_fast(float r) {
  return __fdividef(r, 1.0f + __expf(fminf(-r, 80.0f)));
}
// 16-bit outputs: x * sigmoid(x) = 0.5 x (1 + tanh(x / 2)) with the hardware
// tanh approximation, one special-function op per element instead of two;
// its error (~2^-11 relative) is below the 16-bit output rounding.
__device__ __forceinline__ float silu_tanh(float r) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * r));
  return 0.5f * r * (1.0f + t);
}
template <int DT>
__device__ __forceinline__ float silu_out(float r) {
  return DT == T2SC_DT_F32 ? silu_fast(r) : silu_tanh(r);
}

// Sum over the T lanes of this row's group (T a power of two <= 32; groups
// are aligned lane ranges, so xor partners stay inside the group). R
// independent sums interleaved for shuffle ILP.
template <int R>
__device__ __forceinline__ void group_sum(float (&v)[R], int t) {
  for (int d = t >> 1; d > 0; d >>= 1) {
#pragma unroll
    for (int r = 0; r < R; r++) v[r] += __shfl_xor_sync(0xffffffffu, v[r], d);
  }
}

template <int DT>
__device__ __forceinline__ float ld1(const void *p, int64_t i) {
  if (DT == T2SC_DT_F32) return static_cast<const float *>(p)[i];
  if (DT == T2SC_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}
template <int DT>
__device__ __forceinline__ void st1(void *p, int64_t i, float v) {
  if (DT == T2SC_DT_F32)
    static_cast<float *>(p)[i] = v;
  else if (DT == T2SC_DT_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

// 16-byte chunk <-> E floats.
template <int DT>
struct Vec {
  static constexpr int kElems = DT == T2SC_DT_F32 ? 4 : 8;
  __device__ __forceinline__ static void unpack(const uint4 &u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (DT == T2SC_DT_F32) {
        f[j] = __uint_as_float(w[j]);
      } else if (DT == T2SC_DT_BF16) {
        __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162 *>(&w[j]);
        f[2 * j] = __low2float(p), f[2 * j + 1] = __high2float(p);
      } else {
        __half2 p = *reinterpret_cast<const __half2 *>(&w[j]);
        f[2 * j] = __low2float(p), f[2 * j + 1] = __high2float(p);
      }
    }
  }
  __device__ __forceinline__ static uint4 pack(const float *f) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (DT == T2SC_DT_F32) {
        w[j] = __float_as_uint(f[j]);
      } else if (DT == T2SC_DT_BF16) {
        __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t *>(&p);
      } else {
        __half2 p = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t *>(&p);
      }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

constexpr int kThreads = 256;

// x, y: [rows, chunks] 16-byte chunks (y may alias x: every element is read
// before the same lane writes it). w, b: f32 [c] 16-byte aligned, or null.
template <int DT, int V, int R>
__global__ void __launch_bounds__(kThreads) layernorm_vec_kernel(const uint4 *x, uint4 *y, int64_t rows, int c,
                                                                 int chunks, int t, const float4 *__restrict__ w,
                                                                 const float4 *__restrict__ b, float eps,
                                                                 int silu) {
  constexpr int E = Vec<DT>::kElems;
  const int groups = kThreads / t;
  const int gid = (int)threadIdx.x / t, sub = (int)threadIdx.x % t;
  const int64_t row0 = (int64_t)blockIdx.x * groups * R + gid;
  float v[R][V][E];
  float s[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int64_t row = row0 + (int64_t)r * groups;
#pragma unroll
    for (int q = 0; q < V; q++) {
      const int ch = q * t + sub;
      if (row < rows && ch < chunks) {
        Vec<DT>::unpack(__ldcs(x + row * chunks + ch), v[r][q]);
      } else {
#pragma unroll
        for (int e = 0; e < E; e++) v[r][q][e] = 0.f;
      }
    }
  }
  const float inv_c = 1.0f / (float)c;
#pragma unroll
  for (int r = 0; r < R; r++) {
    s[r] = 0.f;
#pragma unroll
    for (int q = 0; q < V; q++)
#pragma unroll
      for (int e = 0; e < E; e++) s[r] += v[r][q][e];
  }
  group_sum<R>(s, t);
  float mean[R], ss[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    mean[r] = s[r] * inv_c;
    ss[r] = 0.f;
#pragma unroll
    for (int q = 0; q < V; q++) {
      if (q * t + sub < chunks) {
#pragma unroll
        for (int e = 0; e < E; e++) {
          const float d = v[r][q][e] - mean[r];
          ss[r] += d * d;
        }
      }
    }
  }
  group_sum<R>(ss, t);
#pragma unroll
  for (int q = 0; q < V; q++) {
    const int ch = q * t + sub;
    if (ch >= chunks) continue;
    float wq[E], bq[E];
    if (w) {
#pragma unroll
      for (int e4 = 0; e4 < E / 4; e4++) {
        const float4 a = __ldg(w + ch * (E / 4) + e4), o = __ldg(b + ch * (E / 4) + e4);
        wq[4 * e4] = a.x, wq[4 * e4 + 1] = a.y, wq[4 * e4 + 2] = a.z, wq[4 * e4 + 3] = a.w;
        bq[4 * e4] = o.x, bq[4 * e4 + 1] = o.y, bq[4 * e4 + 2] = o.z, bq[4 * e4 + 3] = o.w;
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int64_t row = row0 + (int64_t)r * groups;
      if (row >= rows) continue;
      const float inv_std = 1.0f / sqrtf(ss[r] * inv_c + eps);
      float o[E];
#pragma unroll
      for (int e = 0; e < E; e++) {
        float z = (v[r][q][e] - mean[r]) * inv_std;
        if (w) z = z * wq[e] + bq[e];
        o[e] = silu ? silu_out<DT>(z) : z;
      }
      __stcs(y + row * chunks + ch, Vec<DT>::pack(o));
    }
  }
}

// Any C (<= 1024), any alignment: element granularity, P elements per lane.
template <int DT, int P>
__global__ void __launch_bounds__(kThreads) layernorm_scalar_kernel(const void *x, void *y, int64_t rows, int c,
                                                                    int t, const float *__restrict__ w,
                                                                    const float *__restrict__ b, float eps,
                                                                    int silu) {
  const int groups = kThreads / t;
  const int gid = (int)threadIdx.x / t, sub = (int)threadIdx.x % t;
  const int64_t row = (int64_t)blockIdx.x * groups + gid;
  const bool live = row < rows;  // dead lanes still join the shuffles
  const int64_t base = (live ? row : 0) * c;
  float v[P];
  float s[1] = {0.f};
#pragma unroll
  for (int q = 0; q < P; q++) {
    const int i = q * t + sub;
    v[q] = (live && i < c) ? ld1<DT>(x, base + i) : 0.f;
    s[0] += v[q];
  }
  group_sum<1>(s, t);
  const float mean = s[0] / (float)c;
  float ss[1] = {0.f};
#pragma unroll
  for (int q = 0; q < P; q++) {
    const float d = (q * t + sub < c) ? v[q] - mean : 0.f;
    ss[0] += d * d;
  }
  group_sum<1>(ss, t);
  const float inv_std = 1.0f / sqrtf(ss[0] / (float)c + eps);
  if (!live) return;
#pragma unroll
  for (int q = 0; q < P; q++) {
    const int i = q * t + sub;
    if (i < c) {
      float z = (v[q] - mean) * inv_std;
      if (w) z = z * w[i] + b[i];
      st1<DT>(y, base + i, silu ? silu_out<DT>(z) : z);
    }
  }
}

inline int group_lanes(int units) {
  int t = 1;
  while (t < units && t < 32) t <<= 1;
  return t;
}

template <int DT>
int launch_vec(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w, const float *b, float eps,
               int silu, std::string &err) {
  const int chunks = c / Vec<DT>::kElems;
  const int t = group_lanes(chunks);
  const int per = (chunks + t - 1) / t;  // chunks per lane: 1..8
  const int groups = kThreads / t;
  auto xp = static_cast<const uint4 *>(x);
  auto yp = static_cast<uint4 *>(y);
  auto wp = reinterpret_cast<const float4 *>(w);
  auto bp = reinterpret_cast<const float4 *>(b);
  auto grid = [&](int r) { return (unsigned)((rows + (int64_t)groups * r - 1) / ((int64_t)groups * r)); };
  if (per == 1)
    layernorm_vec_kernel<DT, 1, 8><<<grid(8), kThreads, 0, ctx->stream>>>(xp, yp, rows, c, chunks, t, wp, bp, eps, silu);
  else if (per == 2)
    layernorm_vec_kernel<DT, 2, 4><<<grid(4), kThreads, 0, ctx->stream>>>(xp, yp, rows, c, chunks, t, wp, bp, eps, silu);
  else if (per <= 4)
    layernorm_vec_kernel<DT, 4, 2><<<grid(2), kThreads, 0, ctx->stream>>>(xp, yp, rows, c, chunks, t, wp, bp, eps, silu);
  else
    layernorm_vec_kernel<DT, 8, 1><<<grid(1), kThreads, 0, ctx->stream>>>(xp, yp, rows, c, chunks, t, wp, bp, eps, silu);
  T2SC_LAUNCHED(ctx, "layernorm_vec");
  return T2SC_OK;
}

template <int DT>
int launch_scalar(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w, const float *b,
                  float eps, int silu, std::string &err) {
  const int t = group_lanes(c);
  const int per = (c + t - 1) / t;  // 1..32
  const unsigned grid = (unsigned)((rows + kThreads / t - 1) / (kThreads / t));
#define T2SC_LN_SCALAR(P) layernorm_scalar_kernel<DT, P><<<grid, kThreads, 0, ctx->stream>>>(x, y, rows, c, t, w, b, eps, silu)
  if (per == 1)
    T2SC_LN_SCALAR(1);
  else if (per == 2)
    T2SC_LN_SCALAR(2);
  else if (per <= 4)
    T2SC_LN_SCALAR(4);
  else if (per <= 8)
    T2SC_LN_SCALAR(8);
  else if (per <= 16)
    T2SC_LN_SCALAR(16);
  else
    T2SC_LN_SCALAR(32);
#undef T2SC_LN_SCALAR
  T2SC_LAUNCHED(ctx, "layernorm_scalar");
  return T2SC_OK;
}

}  // namespace

int layernorm_device(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w, const float *b,
                     float eps, int flags, int dtype, std::string &err) {
  if (rows == 0) return T2SC_OK;
  const int silu = (flags & T2SC_SILU) ? 1 : 0;
  const int s = dtype == T2SC_DT_F32 ? 4 : 2;
  const bool vec = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && ((uintptr_t)w % 16 == 0) &&
                   ((uintptr_t)b % 16 == 0) && ((int64_t)c * s) % 16 == 0;
  if (dtype == T2SC_DT_F32)
    return vec ? launch_vec<T2SC_DT_F32>(ctx, x, y, rows, c, w, b, eps, silu, err)
               : launch_scalar<T2SC_DT_F32>(ctx, x, y, rows, c, w, b, eps, silu, err);
  if (dtype == T2SC_DT_BF16)
    return vec ? launch_vec<T2SC_DT_BF16>(ctx, x, y, rows, c, w, b, eps, silu, err)
               : launch_scalar<T2SC_DT_BF16>(ctx, x, y, rows, c, w, b, eps, silu, err);
  return vec ? launch_vec<T2SC_DT_F16>(ctx, x, y, rows, c, w, b, eps, silu, err)
             : launch_scalar<T2SC_DT_F16>(ctx, x, y, rows, c, w, b, eps, silu, err);
}

}  // namespace t2sc
