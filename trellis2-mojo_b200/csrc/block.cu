// The decoder's up block, SparseResBlockC2S3d
// (trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:67-133), on the device:
//
//   subdiv = to_subdiv(x)                       (pred_subdiv; else given)
//   h  = SiLU(LN1(x))                           LayerNorm affine, eps 1e-6
//   h  = conv1(h)                               C -> 8*Cout
//   h  = C2S(h, subdiv > 0)                     children, feats slice c*Cout
//   x2 = C2S(x, subdiv > 0)                     feats slice c*(C/8)
//   h  = SiLU(LN2(h))                           LayerNorm no affine, eps 1e-6
//   out = conv2(h) + repeat_interleave(x2, Cout/(C/8))
//
// Every step is a libt2sc kernel on the context's stream; the skip term
// (the C2S of x repeated along channels) is gathered straight from x into
// the residual operand of conv2's epilogue.
#include <vector>

#include "internal.h"

struct t2sc_c2s_block {
  t2sc_ctx *ctx = nullptr;
  int channels = 0, out_channels = 0, pred_subdiv = 0, dtype = 0;
  float *d_norm1 = nullptr;  // [2, C]: weight then bias
  t2sc_conv *conv1 = nullptr, *conv2 = nullptr, *to_subdiv = nullptr;
};

namespace {

constexpr float kBlockEps = 1e-6f;  // both norms (sparse_unet_vae.mojo:78-79)

// skip[e, o] = x[parent[e], subidx[e] * (C/8) + o / k] with k = Cout / (C/8):
// the C2S unfold of x followed by repeat_interleave along channels.
template <typename T>
__global__ void c2s_skip_kernel(const T *__restrict__ x, int c, const int32_t *__restrict__ parent,
                                const int32_t *__restrict__ subidx, int64_t m, int cout, T *__restrict__ skip) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * cout) return;
  const int64_t e = i / cout;
  const int o = (int)(i % cout), c8 = c / 8, k = cout / c8;
  skip[i] = x[(int64_t)parent[e] * c + (int64_t)subidx[e] * c8 + o / k];
}

int fail(t2sc_ctx *ctx, int code, const std::string &msg) {
  ctx->last_error = msg;
  return code;
}

}  // namespace

extern "C" {

int t2sc_c2s_block_create(t2sc_ctx *ctx, int channels, int out_channels, int pred_subdiv, const float *norm1_w,
                          const float *norm1_b, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                          const float *conv2_b, const float *to_subdiv_w, const float *to_subdiv_b, int dtype,
                          t2sc_c2s_block **out) {
  if (!ctx || !out) return T2SC_ERR_INVALID;
  *out = nullptr;
  if (channels < 8 || channels % 8 || out_channels < 1 || out_channels % (channels / 8) || channels > 1024 ||
      out_channels > 1024)
    return fail(ctx, T2SC_ERR_INVALID,
                "c2s block: need C % 8 == 0, Cout a multiple of C/8, both <= 1024 (LayerNorm width)");
  if (!norm1_w || !norm1_b || !conv1_w || !conv2_w || (pred_subdiv && !to_subdiv_w))
    return fail(ctx, T2SC_ERR_INVALID, "c2s block: null weight");
  std::unique_ptr<t2sc_c2s_block, int (*)(t2sc_c2s_block *)> b(new t2sc_c2s_block(), t2sc_c2s_block_destroy);
  b->ctx = ctx;
  b->channels = channels;
  b->out_channels = out_channels;
  b->pred_subdiv = pred_subdiv ? 1 : 0;
  b->dtype = dtype;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  std::vector<float> wb(2 * (size_t)channels);
  for (int i = 0; i < channels; i++) wb[i] = norm1_w[i], wb[channels + i] = norm1_b[i];
  int rc = T2SC_OK;
  if (cudaMalloc((void **)&b->d_norm1, wb.size() * 4) != cudaSuccess ||
      cudaMemcpy(b->d_norm1, wb.data(), wb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(ctx, T2SC_ERR_OOM, "c2s block: norm weights");
  if (rc == T2SC_OK)
    rc = t2sc_conv_create(ctx, conv1_w, conv1_b, 8 * out_channels, 3, 3, 3, channels, 1, dtype, &b->conv1);
  if (rc == T2SC_OK)
    rc = t2sc_conv_create(ctx, conv2_w, conv2_b, out_channels, 3, 3, 3, out_channels, 1, dtype, &b->conv2);
  if (rc == T2SC_OK && pred_subdiv)
    rc = t2sc_linear_create(ctx, to_subdiv_w, to_subdiv_b, 8, channels, dtype, &b->to_subdiv);
  if (prev >= 0) cudaSetDevice(prev);
  if (rc != T2SC_OK) return rc;
  *out = b.release();
  return T2SC_OK;
}

int t2sc_c2s_block_destroy(t2sc_c2s_block *b) {
  if (!b) return T2SC_OK;
  t2sc_conv_destroy(b->conv1);
  t2sc_conv_destroy(b->conv2);
  t2sc_conv_destroy(b->to_subdiv);
  if (b->d_norm1) cudaFree(b->d_norm1);
  delete b;
  return T2SC_OK;
}

int t2sc_c2s_block_forward_device(t2sc_c2s_block *b, t2sc_coords *coords, const void *x, float *subdiv,
                                  int32_t *out_coords, void *out_feats, int64_t *m, t2sc_coords **out_child) {
  if (!b || !coords || !m) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = b->ctx;
  if (out_child) *out_child = nullptr;
  *m = 0;
  if (coords->ctx != ctx) return fail(ctx, T2SC_ERR_INVALID, "c2s block: coords of another context");
  if (coords->n_targets != coords->n || coords->target_begin != 0)
    return fail(ctx, T2SC_ERR_INVALID, "c2s block: coordinates with halo rows are not supported");
  const int64_t n = coords->n;
  if (n == 0) return T2SC_OK;
  if (!x || !subdiv || !out_coords || !out_feats) return fail(ctx, T2SC_ERR_INVALID, "c2s block: null buffer");
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  std::string &err = ctx->last_error;
  cudaStream_t st = ctx->stream;
  const int C = b->channels, Co = b->out_channels, dt = b->dtype;
  const size_t es = dt == T2SC_DT_F32 ? 4 : 2;
  void *h1 = nullptr, *h2 = nullptr, *h3 = nullptr, *skip = nullptr, *sub16 = nullptr;
  int32_t *par = nullptr, *sidx = nullptr;
  t2sc_coords *child = nullptr;
  int64_t mm = 0;
  auto body = [&]() -> int {
    T2SC_CUDA(cudaMallocAsync(&h1, (size_t)n * C * es, st), "c2s scratch");
    T2SC_CUDA(cudaMallocAsync(&h2, (size_t)n * 8 * Co * es, st), "c2s scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&par, (size_t)n * 8 * 4, st), "c2s scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&sidx, (size_t)n * 8 * 4, st), "c2s scratch");
    int rc;
    if (b->pred_subdiv) {  // subdiv = to_subdiv(x), kept in f32 for the > 0 test
      if (dt == T2SC_DT_F32) {
        if ((rc = t2sc_linear_forward_device(b->to_subdiv, x, subdiv, n, 0, nullptr)) != T2SC_OK) return rc;
      } else {
        T2SC_CUDA(cudaMallocAsync(&sub16, (size_t)n * 8 * es, st), "c2s scratch");
        if ((rc = t2sc_linear_forward_device(b->to_subdiv, x, sub16, n, 0, nullptr)) != T2SC_OK) return rc;
        if ((rc = t2sc::dtype_to_f32(ctx, sub16, subdiv, n * 8, dt)) != T2SC_OK) return rc;
      }
    }
    if ((rc = t2sc_layernorm_device(ctx, x, h1, n, C, b->d_norm1, b->d_norm1 + C, kBlockEps, T2SC_SILU, dt)) !=
        T2SC_OK)
      return rc;
    if ((rc = t2sc_conv_forward_device(b->conv1, coords, h1, h2, 0, nullptr)) != T2SC_OK) return rc;
    // children of the positive entries and their conv1 channel slices
    T2SC_CUDA(cudaMallocAsync(&h3, (size_t)n * 8 * Co * es, st), "c2s scratch");
    if ((rc = t2sc::subdivide_device(ctx, coords->d_coords, n, subdiv, T2SC_SUB_POSITIVE, h2, Co, T2SC_FEATS_C2S,
                                     dt, out_coords, h3, par, sidx, &mm, err)) != T2SC_OK)
      return rc;
    if (mm == 0) return T2SC_OK;
    T2SC_CUDA(cudaMallocAsync(&skip, (size_t)mm * Co * es, st), "c2s scratch");
    const unsigned blocks = (unsigned)((mm * Co + 255) / 256);
    if (es == 4)
      c2s_skip_kernel<float><<<blocks, 256, 0, st>>>((const float *)x, C, par, sidx, mm, Co, (float *)skip);
    else
      c2s_skip_kernel<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)x, C, par, sidx, mm, Co,
                                                        (uint16_t *)skip);
    T2SC_LAUNCHED(ctx, "c2s_skip");
    if ((rc = t2sc_layernorm_device(ctx, h3, h3, mm, Co, nullptr, nullptr, kBlockEps, T2SC_SILU, dt)) != T2SC_OK)
      return rc;
    if ((rc = t2sc_coords_create_device(ctx, out_coords, mm, &child)) != T2SC_OK) return rc;
    if ((rc = t2sc_conv_forward_device(b->conv2, child, h3, out_feats, T2SC_RESIDUAL, skip)) != T2SC_OK) return rc;
    return T2SC_OK;
  };
  int rc = body();
  for (void *p : {h1, h2, h3, skip, sub16, (void *)par, (void *)sidx})
    if (p) cudaFreeAsync(p, st);
  if (rc == T2SC_OK) {
    *m = mm;
    if (out_child)
      *out_child = child;
    else
      t2sc_coords_destroy(child);
  } else {
    t2sc_coords_destroy(child);
  }
  if (prev >= 0) cudaSetDevice(prev);
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// SparseConvNeXtBlock3d (sparse_unet_vae.mojo:40-64):
//   y = lin2(SiLU(lin1(LN(conv(x))))) + x,  LN affine eps 1e-6.
// Four kernels on the context's stream: the conv, LayerNorm in place, lin1
// with SiLU fused, lin2 with the residual x fused into its epilogue.

struct t2sc_convnext_block {
  t2sc_ctx *ctx = nullptr;
  int channels = 0, hidden = 0, dtype = 0;
  float *d_norm = nullptr;  // [2, C]
  t2sc_conv *conv = nullptr, *lin1 = nullptr, *lin2 = nullptr;
};

extern "C" {

int t2sc_convnext_block_create(t2sc_ctx *ctx, int channels, int hidden, const float *conv_w, const float *conv_b,
                               const float *norm_w, const float *norm_b, const float *lin1_w, const float *lin1_b,
                               const float *lin2_w, const float *lin2_b, int dtype, t2sc_convnext_block **out) {
  if (!ctx || !out) return T2SC_ERR_INVALID;
  *out = nullptr;
  if (channels < 1 || channels > 1024 || hidden < 1)
    return fail(ctx, T2SC_ERR_INVALID, "convnext block: need 1 <= C <= 1024 (LayerNorm width) and hidden >= 1");
  if (!conv_w || !norm_w || !norm_b || !lin1_w || !lin2_w)
    return fail(ctx, T2SC_ERR_INVALID, "convnext block: null weight");
  std::unique_ptr<t2sc_convnext_block, int (*)(t2sc_convnext_block *)> b(new t2sc_convnext_block(),
                                                                         t2sc_convnext_block_destroy);
  b->ctx = ctx;
  b->channels = channels;
  b->hidden = hidden;
  b->dtype = dtype;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  std::vector<float> wb(2 * (size_t)channels);
  for (int i = 0; i < channels; i++) wb[i] = norm_w[i], wb[channels + i] = norm_b[i];
  int rc = T2SC_OK;
  if (cudaMalloc((void **)&b->d_norm, wb.size() * 4) != cudaSuccess ||
      cudaMemcpy(b->d_norm, wb.data(), wb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(ctx, T2SC_ERR_OOM, "convnext block: norm weights");
  if (rc == T2SC_OK) rc = t2sc_conv_create(ctx, conv_w, conv_b, channels, 3, 3, 3, channels, 1, dtype, &b->conv);
  if (rc == T2SC_OK) rc = t2sc_linear_create(ctx, lin1_w, lin1_b, hidden, channels, dtype, &b->lin1);
  if (rc == T2SC_OK) rc = t2sc_linear_create(ctx, lin2_w, lin2_b, channels, hidden, dtype, &b->lin2);
  if (prev >= 0) cudaSetDevice(prev);
  if (rc != T2SC_OK) return rc;
  *out = b.release();
  return T2SC_OK;
}

int t2sc_convnext_block_destroy(t2sc_convnext_block *b) {
  if (!b) return T2SC_OK;
  t2sc_conv_destroy(b->conv);
  t2sc_conv_destroy(b->lin1);
  t2sc_conv_destroy(b->lin2);
  if (b->d_norm) cudaFree(b->d_norm);
  delete b;
  return T2SC_OK;
}

int t2sc_convnext_block_forward_device(t2sc_convnext_block *b, t2sc_coords *coords, const void *x, void *y) {
  if (!b || !coords) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = b->ctx;
  if (coords->ctx != ctx) return fail(ctx, T2SC_ERR_INVALID, "convnext block: coords of another context");
  if (coords->n_targets != coords->n || coords->target_begin != 0)
    return fail(ctx, T2SC_ERR_INVALID, "convnext block: coordinates with halo rows are not supported");
  const int64_t n = coords->n;
  if (n == 0) return T2SC_OK;
  if (!x || !y || x == y) return fail(ctx, T2SC_ERR_INVALID, "convnext block: null or aliased buffers");
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  std::string &err = ctx->last_error;
  cudaStream_t st = ctx->stream;
  const size_t es = b->dtype == T2SC_DT_F32 ? 4 : 2;
  void *h1 = nullptr, *h2 = nullptr;
  auto body = [&]() -> int {
    T2SC_CUDA(cudaMallocAsync(&h1, (size_t)n * b->channels * es, st), "convnext scratch");
    T2SC_CUDA(cudaMallocAsync(&h2, (size_t)n * b->hidden * es, st), "convnext scratch");
    int rc;
    if ((rc = t2sc_conv_forward_device(b->conv, coords, x, h1, 0, nullptr)) != T2SC_OK) return rc;
    if ((rc = t2sc_layernorm_device(ctx, h1, h1, n, b->channels, b->d_norm, b->d_norm + b->channels, kBlockEps, 0,
                                    b->dtype)) != T2SC_OK)
      return rc;
    if ((rc = t2sc_linear_forward_device(b->lin1, h1, h2, n, T2SC_SILU, nullptr)) != T2SC_OK) return rc;
    return t2sc_linear_forward_device(b->lin2, h2, y, n, T2SC_RESIDUAL, x);
  };
  int rc = body();
  if (h1) cudaFreeAsync(h1, st);
  if (h2) cudaFreeAsync(h2, st);
  if (prev >= 0) cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
