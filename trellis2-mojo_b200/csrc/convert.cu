// f32 <-> 16-bit conversions for the host-pointer entry points (round to
// nearest even, the hardware conversion).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace t2sc {
namespace {
template <int DT>
__global__ void to16_kernel(const float *__restrict__ in, uint16_t *__restrict__ out, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (DT == T2SC_DT_BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(in[i]);
    out[i] = *reinterpret_cast<uint16_t *>(&h);
  } else {
    __half h = __float2half_rn(in[i]);
    out[i] = *reinterpret_cast<uint16_t *>(&h);
  }
}
template <int DT>
__global__ void from16_kernel(const uint16_t *__restrict__ in, float *__restrict__ out, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint16_t b = in[i];
  if (DT == T2SC_DT_BF16)
    out[i] = __bfloat162float(*reinterpret_cast<__nv_bfloat16 *>(&b));
  else
    out[i] = __half2float(*reinterpret_cast<__half *>(&b));
}
inline unsigned nb(int64_t n) { return (unsigned)((n + 255) / 256); }
}  // namespace

int f32_to_dtype(t2sc_ctx *ctx, const float *in, void *out, int64_t count, int dtype) {
  std::string &err = ctx->last_error;
  if (count <= 0) return T2SC_OK;
  if (dtype == T2SC_DT_F32) {
    T2SC_CUDA(cudaMemcpyAsync(out, in, count * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy");
    return T2SC_OK;
  }
  if (dtype == T2SC_DT_BF16)
    to16_kernel<T2SC_DT_BF16><<<nb(count), 256, 0, ctx->stream>>>(in, (uint16_t *)out, count);
  else
    to16_kernel<T2SC_DT_F16><<<nb(count), 256, 0, ctx->stream>>>(in, (uint16_t *)out, count);
  T2SC_LAUNCHED(ctx, "to16");
  return T2SC_OK;
}

int dtype_to_f32(t2sc_ctx *ctx, const void *in, float *out, int64_t count, int dtype) {
  std::string &err = ctx->last_error;
  if (count <= 0) return T2SC_OK;
  if (dtype == T2SC_DT_F32) {
    T2SC_CUDA(cudaMemcpyAsync(out, in, count * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy");
    return T2SC_OK;
  }
  if (dtype == T2SC_DT_BF16)
    from16_kernel<T2SC_DT_BF16><<<nb(count), 256, 0, ctx->stream>>>((const uint16_t *)in, out, count);
  else
    from16_kernel<T2SC_DT_F16><<<nb(count), 256, 0, ctx->stream>>>((const uint16_t *)in, out, count);
  T2SC_LAUNCHED(ctx, "from16");
  return T2SC_OK;
}
}  // namespace t2sc
