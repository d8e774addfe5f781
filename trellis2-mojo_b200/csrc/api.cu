// C-ABI entry points of libt2sc (declared in include/t2sc.h).
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <new>
#include <vector>

#include "internal.h"

using namespace t2sc;

namespace {

// Makes the context's device current for the duration of a call and
// restores the caller's device afterwards.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int fail(t2sc_ctx *ctx, int code, const std::string &msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

size_t elem_size(int dtype) { return dtype == T2SC_DT_F32 ? 4 : 2; }

// Stream-ordered temporary device buffer.
struct DevBuf {
  void *p = nullptr;
  cudaStream_t st = nullptr;
  DevBuf() = default;
  DevBuf(const DevBuf &) = delete;
  ~DevBuf() {
    if (p) cudaFreeAsync(p, st);
  }
  int alloc(t2sc_ctx *ctx, size_t bytes) {
    st = ctx->stream;
    std::string &err = ctx->last_error;
    T2SC_CUDA(cudaMallocAsync(&p, bytes ? bytes : 16, st), "device buffer");
    return T2SC_OK;
  }
};

#define T2SC_TRY(expr)                   \
  do {                                   \
    int _rc = (expr);                    \
    if (_rc != T2SC_OK) return _rc;      \
  } while (0)

// Runs an entry point's body; C++ exceptions never cross the C ABI.
template <class F>
int guarded(t2sc_ctx *ctx, F &&body) {
  try {
    return body();
  } catch (const std::bad_alloc &) {
    return fail(ctx, T2SC_ERR_OOM, "host allocation failed");
  } catch (...) {
    return fail(ctx, T2SC_ERR_INVALID, "unexpected exception");
  }
}

int check_sync(t2sc_ctx *ctx) {
  std::string &err = ctx->last_error;
  T2SC_CUDA(cudaStreamSynchronize(ctx->stream), "stream synchronize");
  int flags = 0;
  T2SC_TRY(read_dev_err(ctx, &flags));
  if (flags & kDevErrTimeout)
    return fail(ctx, T2SC_ERR_TIMEOUT, "a bounded device wait timed out; results of the last call are invalid");
  if (flags) return fail(ctx, T2SC_ERR_INVALID, "device error flags set: " + std::to_string(flags));
  return T2SC_OK;
}

}  // namespace

int t2sc::read_dev_err(t2sc_ctx *ctx, int *flags) {
  std::string &err = ctx->last_error;
  int h = 0;
  T2SC_CUDA(cudaMemcpyAsync(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream), "read error flags");
  T2SC_CUDA(cudaStreamSynchronize(ctx->stream), "read error flags");
  if (h) T2SC_CUDA(cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream), "clear error flags");
  *flags = h;
  return T2SC_OK;
}

extern "C" {

const char *t2sc_version(void) { return "t2sc 0.1 sm_100a"; }

int t2sc_ctx_create(int device, t2sc_ctx **out) {
  if (!out) return T2SC_ERR_INVALID;
  *out = nullptr;
  return guarded(nullptr, [&]() -> int {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return T2SC_ERR_CUDA;
    DeviceGuard g(device);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return T2SC_ERR_CUDA;
    if (prop.major != 10) return T2SC_ERR_UNSUPPORTED;  // built for sm_100a only
    std::unique_ptr<t2sc_ctx> ctx(new t2sc_ctx());
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess) return T2SC_ERR_CUDA;
    // keep the device's stream-ordered pool warm: scratch freed by one call
    // is reused by the next instead of being unmapped at every synchronise
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    ctx->stream = ctx->own_stream;
    if (cudaMalloc((void **)&ctx->d_err, sizeof(int)) != cudaSuccess) return T2SC_ERR_OOM;
    if (cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess) return T2SC_ERR_CUDA;
    *out = ctx.release();
    return T2SC_OK;
  });
}

int t2sc_ctx_destroy(t2sc_ctx *ctx) {
  if (!ctx) return T2SC_OK;
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (void *p : ctx->stage)
    if (p) cudaFree(p);
  for (auto &kv : ctx->id_maps) free_map(kv.second);
  cudaFree(ctx->d_err);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  if (ctx->up_stream) cudaStreamDestroy(ctx->up_stream);
  if (ctx->down_stream) cudaStreamDestroy(ctx->down_stream);
  delete ctx;
  return T2SC_OK;
}

int t2sc_ctx_set_stream(t2sc_ctx *ctx, void *stream) {
  if (!ctx) return T2SC_ERR_INVALID;
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return T2SC_OK;
}

int t2sc_ctx_synchronize(t2sc_ctx *ctx) {
  if (!ctx) return T2SC_ERR_INVALID;
  DeviceGuard g(ctx->device);
  return check_sync(ctx);
}

const char *t2sc_last_error(const t2sc_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int t2sc_ctx_launch_count(const t2sc_ctx *ctx, int64_t *count) {
  if (!ctx || !count) return T2SC_ERR_INVALID;
  *count = ctx->launches;
  return T2SC_OK;
}

// ------------------------------- coordinates -------------------------------

static int coords_create_impl(t2sc_ctx *ctx, const int32_t *coords, int64_t n, int64_t n_targets, bool on_device,
                              t2sc_coords **out, int64_t target_begin = 0) {
  if (!ctx || !out) return T2SC_ERR_INVALID;
  *out = nullptr;
  if (n < 0 || (n > 0 && !coords)) return fail(ctx, T2SC_ERR_INVALID, "coords: bad pointer or count");
  if (target_begin < 0 || n_targets < 0 || target_begin + n_targets > n)
    return fail(ctx, T2SC_ERR_INVALID, "coords: target rows must lie in [0, n)");
  if (n >= (int64_t(1) << 31)) return fail(ctx, T2SC_ERR_UNSUPPORTED, "coords: more than 2^31-1 rows");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    std::string &err = ctx->last_error;
    std::unique_ptr<t2sc_coords> c(new t2sc_coords());
    c->ctx = ctx;
    c->n = n;
    c->n_targets = n_targets;
    c->target_begin = target_begin;
    T2SC_CUDA(cudaMallocAsync((void **)&c->d_coords, (size_t)(n > 0 ? n : 1) * 16, ctx->stream), "coords");
    if (n > 0)
      T2SC_CUDA(cudaMemcpyAsync(c->d_coords, coords, (size_t)n * 16,
                                on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream),
                "coords upload");
    int rc = build_hash(c.get(), err);
    if (rc != T2SC_OK) {
      t2sc_coords_destroy(c.release());
      return rc;
    }
    *out = c.release();
    return T2SC_OK;
  });
}

int t2sc_coords_create(t2sc_ctx *ctx, const int32_t *coords, int64_t n, t2sc_coords **out) {
  return coords_create_impl(ctx, coords, n, n, false, out);
}
int t2sc_coords_create_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, t2sc_coords **out) {
  return coords_create_impl(ctx, coords, n, n, true, out);
}
int t2sc_coords_create_halo(t2sc_ctx *ctx, const int32_t *coords, int64_t n, int64_t n_targets, int on_device,
                            t2sc_coords **out) {
  return coords_create_impl(ctx, coords, n, n_targets, on_device != 0, out);
}

int t2sc_coords_create_range(t2sc_ctx *ctx, const int32_t *coords, int64_t n, int64_t target_begin,
                             int64_t target_end, int on_device, t2sc_coords **out) {
  return coords_create_impl(ctx, coords, n, target_end - target_begin, on_device != 0, out, target_begin);
}

int t2sc_coords_destroy(t2sc_coords *c) {
  if (!c) return T2SC_OK;
  DeviceGuard g(c->ctx->device);
  // stream-ordered release: work already queued on the context's stream
  // that reads these buffers still runs first, and nothing synchronises
  for (auto &kv : c->maps) free_map(kv.second);
  for (auto &kv : c->chain_plans)
    for (auto &sl : kv.second) {
      t2sc_coords_destroy(sl.all);
      t2sc_coords_destroy(sl.own);
    }
  cudaFreeAsync(c->d_coords, c->ctx->stream);
  cudaFreeAsync(c->d_slots, c->ctx->stream);
  delete c;
  return T2SC_OK;
}

int t2sc_coords_count(const t2sc_coords *c, int64_t *n) {
  if (!c || !n) return T2SC_ERR_INVALID;
  *n = c->n_targets;
  return T2SC_OK;
}

static int kernel_ok(t2sc_ctx *ctx, int kd, int kh, int kw, int dil) {
  if (kd < 1 || kh < 1 || kw < 1 || kd * kh * kw > kMaxK)
    return fail(ctx, T2SC_ERR_UNSUPPORTED, "kernel volume must be 1..32");
  if (dil < 1 || dil > 512) return fail(ctx, T2SC_ERR_INVALID, "dilation must be >= 1");
  return T2SC_OK;
}

int t2sc_coords_build_map(t2sc_coords *c, int kd, int kh, int kw, int dil, int64_t *n_edges) {
  if (!c) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = c->ctx;
  T2SC_TRY(kernel_ok(ctx, kd, kh, kw, dil));
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    t2sc_map *m = nullptr;
    T2SC_TRY(build_map(c, kd, kh, kw, dil, &m, ctx->last_error));
    int64_t e = 0;
    if (n_edges) T2SC_TRY(map_edges(m, &e, ctx->last_error));
    if (n_edges) *n_edges = e;
    return T2SC_OK;
  });
}

int t2sc_neighbor_map_export(t2sc_coords *c, int kd, int kh, int kw, int dil, int64_t *src, int64_t *tgt,
                             int64_t *kidx, int64_t cap, int64_t *n_edges) {
  if (!c || !n_edges) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = c->ctx;
  T2SC_TRY(kernel_ok(ctx, kd, kh, kw, dil));
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    t2sc_map *m = nullptr;
    T2SC_TRY(build_map(c, kd, kh, kw, dil, &m, ctx->last_error));
    T2SC_TRY(map_edges(m, n_edges, ctx->last_error));
    if (m->n_edges > cap) return fail(ctx, T2SC_ERR_CAPACITY, "edge buffers too small");
    if (m->n_edges > 0 && (!src || !tgt || !kidx)) return fail(ctx, T2SC_ERR_INVALID, "null edge buffer");
    T2SC_TRY(export_edges(c, m, src, tgt, kidx, ctx->last_error));
    return check_sync(ctx);
  });
}

int t2sc_csr_export(t2sc_coords *c, int kd, int kh, int kw, int dil, int64_t *row_start, int64_t *src_s,
                    int64_t *kidx_s, int64_t cap, int64_t *n_edges) {
  if (!c || !n_edges || !row_start) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = c->ctx;
  T2SC_TRY(kernel_ok(ctx, kd, kh, kw, dil));
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    t2sc_map *m = nullptr;
    T2SC_TRY(build_map(c, kd, kh, kw, dil, &m, ctx->last_error));
    T2SC_TRY(map_edges(m, n_edges, ctx->last_error));
    if (m->n_edges > cap) return fail(ctx, T2SC_ERR_CAPACITY, "edge buffers too small");
    if (m->n_edges > 0 && (!src_s || !kidx_s)) return fail(ctx, T2SC_ERR_INVALID, "null edge buffer");
    T2SC_TRY(export_csr(c, m, row_start, src_s, kidx_s, ctx->last_error));
    return check_sync(ctx);
  });
}

// ---------------------------------- conv ----------------------------------

int t2sc_conv_create(t2sc_ctx *ctx, const float *weight, const float *bias, int co, int kd, int kh, int kw, int ci,
                     int dilation, int dtype, t2sc_conv **out) {
  if (!ctx || !out) return T2SC_ERR_INVALID;
  *out = nullptr;
  T2SC_TRY(kernel_ok(ctx, kd, kh, kw, dilation));
  if (!weight || co <= 0 || ci <= 0) return fail(ctx, T2SC_ERR_INVALID, "conv: need weight and positive Co, Ci");
  if (dtype != T2SC_DT_F32 && dtype != T2SC_DT_F16 && dtype != T2SC_DT_BF16)
    return fail(ctx, T2SC_ERR_INVALID, "conv: unknown dtype");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    std::string &err = ctx->last_error;
    std::unique_ptr<t2sc_conv> cv(new t2sc_conv());
    cv->ctx = ctx;
    cv->co = co;
    cv->ci = ci;
    cv->kd = kd;
    cv->kh = kh;
    cv->kw = kw;
    cv->kvol = kd * kh * kw;
    cv->dilation = dilation;
    cv->dtype = dtype;
    cv->has_bias = bias != nullptr;
    std::vector<float> b(co, 0.0f);
    if (bias)
      for (int o = 0; o < co; o++) b[o] = bias[o];
    int rc;
    if ((rc = t2sc::cuda_status(cudaMalloc((void **)&cv->d_bias, co * sizeof(float)), err, "bias")) != T2SC_OK ||
        (rc = t2sc::cuda_status(cudaMemcpy(cv->d_bias, b.data(), co * sizeof(float), cudaMemcpyHostToDevice), err,
                                "bias upload")) != T2SC_OK) {
      t2sc_conv_destroy(cv.release());
      return rc;
    }
    // tensor-core kernel: 16-byte row vectors (Ci % 8 for 16-bit, Ci % 4
    // for f32) and N tiles of 16 output channels; the CUDA-core kernel
    // covers every other shape
    cv->tc_path = (co % 16 == 0 && ci % (dtype == T2SC_DT_F32 ? 4 : 8) == 0) ? 1 : 0;
    rc = cv->tc_path ? conv_tc_prepare(cv.get(), weight, err) : conv_simt_prepare(cv.get(), weight, err);
    if (rc != T2SC_OK) {
      t2sc_conv_destroy(cv.release());
      return rc;
    }
    *out = cv.release();
    return T2SC_OK;
  });
}

int t2sc_conv_destroy(t2sc_conv *cv) {
  if (!cv) return T2SC_OK;
  DeviceGuard g(cv->ctx->device);
  cudaStreamSynchronize(cv->ctx->stream);
  cudaFree(cv->d_bias);
  cudaFree(cv->d_wtc);
  cudaFree(cv->d_w_simt);
  cudaFree(cv->d_w_lo);
  delete cv;
  return T2SC_OK;
}

static int forward_device_impl(t2sc_conv *cv, t2sc_coords *c, const void *x, void *y, int flags,
                               const void *residual) {
  t2sc_ctx *ctx = cv->ctx;
  if (c->ctx != ctx) return fail(ctx, T2SC_ERR_INVALID, "conv and coords belong to different contexts");
  if (flags & ~(T2SC_SILU | T2SC_RESIDUAL)) return fail(ctx, T2SC_ERR_INVALID, "unknown flags");
  if ((flags & T2SC_RESIDUAL) && !residual) return fail(ctx, T2SC_ERR_INVALID, "RESIDUAL flag without residual");
  if (c->n > 0 && (!x || !y)) return fail(ctx, T2SC_ERR_INVALID, "null feature buffer");
  t2sc_map *m = nullptr;
  T2SC_TRY(build_map(c, cv->kd, cv->kh, cv->kw, cv->dilation, &m, ctx->last_error));
  return cv->tc_path ? conv_tc_launch(cv, m, x, y, flags, residual, ctx->last_error)
                     : conv_simt_launch(cv, m, x, y, flags, residual, ctx->last_error);
}

int t2sc_linear_create(t2sc_ctx *ctx, const float *weight, const float *bias, int co, int ci, int dtype,
                       t2sc_conv **out) {
  // [Co, Ci] is the [Co, 1, 1, 1, Ci] conv weight
  return t2sc_conv_create(ctx, weight, bias, co, 1, 1, 1, ci, 1, dtype, out);
}

int t2sc_linear_forward_device(t2sc_conv *lin, const void *x, void *y, int64_t rows, int flags,
                               const void *residual) {
  if (!lin) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = lin->ctx;
  if (lin->kvol != 1) return fail(ctx, T2SC_ERR_INVALID, "linear: handle is not a linear layer (kernel volume != 1)");
  if (rows < 0 || rows > INT32_MAX) return fail(ctx, T2SC_ERR_INVALID, "linear: rows must be in [0, 2^31)");
  if (flags & ~(T2SC_SILU | T2SC_RESIDUAL)) return fail(ctx, T2SC_ERR_INVALID, "unknown flags");
  if ((flags & T2SC_RESIDUAL) && !residual) return fail(ctx, T2SC_ERR_INVALID, "RESIDUAL flag without residual");
  if (rows > 0 && (!x || !y)) return fail(ctx, T2SC_ERR_INVALID, "null feature buffer");
  if (rows > 0 && x == y) return fail(ctx, T2SC_ERR_INVALID, "linear: y must not alias x");
  if (rows == 0) return T2SC_OK;
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    // identity map of this row count: built once per context (stream-ordered,
    // no synchronisation) and shared by all linear layers
    t2sc_map *&im = ctx->id_maps[rows];
    if (!im) T2SC_TRY(build_identity_map(ctx, rows, &im, ctx->last_error));
    return lin->tc_path ? conv_tc_launch(lin, im, x, y, flags, residual, ctx->last_error)
                        : conv_simt_launch(lin, im, x, y, flags, residual, ctx->last_error);
  });
}

int t2sc_conv_forward_device(t2sc_conv *cv, t2sc_coords *c, const void *x, void *y, int flags,
                             const void *residual) {
  if (!cv || !c) return T2SC_ERR_INVALID;
  return guarded(cv->ctx, [&]() -> int {
    DeviceGuard g(cv->ctx->device);
    return forward_device_impl(cv, c, x, y, flags, residual);
  });
}

// Host f32 [count] -> device buffer of `dtype` (staging through `tmp32`).
static int upload_as(t2sc_ctx *ctx, const float *h, int64_t count, int dtype, DevBuf &dst) {
  std::string &err = ctx->last_error;
  T2SC_TRY(dst.alloc(ctx, count * elem_size(dtype)));
  if (dtype == T2SC_DT_F32) {
    T2SC_CUDA(cudaMemcpyAsync(dst.p, h, count * 4, cudaMemcpyHostToDevice, ctx->stream), "upload");
    return T2SC_OK;
  }
  DevBuf tmp;
  T2SC_TRY(tmp.alloc(ctx, count * 4));
  T2SC_CUDA(cudaMemcpyAsync(tmp.p, h, count * 4, cudaMemcpyHostToDevice, ctx->stream), "upload");
  return f32_to_dtype(ctx, (const float *)tmp.p, dst.p, count, dtype);
}

static int download_as(t2sc_ctx *ctx, const void *d, int64_t count, int dtype, float *h) {
  std::string &err = ctx->last_error;
  if (dtype == T2SC_DT_F32) {
    T2SC_CUDA(cudaMemcpyAsync(h, d, count * 4, cudaMemcpyDeviceToHost, ctx->stream), "download");
    return T2SC_OK;
  }
  DevBuf tmp;
  T2SC_TRY(tmp.alloc(ctx, count * 4));
  T2SC_TRY(dtype_to_f32(ctx, d, (float *)tmp.p, count, dtype));
  T2SC_CUDA(cudaMemcpyAsync(h, tmp.p, count * 4, cudaMemcpyDeviceToHost, ctx->stream), "download");
  return T2SC_OK;
}

int t2sc_conv_forward(t2sc_conv *cv, t2sc_coords *c, const float *x, float *y, int flags, const float *residual) {
  if (!cv || !c) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = cv->ctx;
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    const int64_t n = c->n_targets, n_src = c->n;
    if (n == 0) return T2SC_OK;
    if (!x || !y) return fail(ctx, T2SC_ERR_INVALID, "null feature buffer");
    if ((flags & T2SC_RESIDUAL) && !residual) return fail(ctx, T2SC_ERR_INVALID, "RESIDUAL flag without residual");
    DevBuf dx, dy, dr;
    T2SC_TRY(upload_as(ctx, x, n_src * cv->ci, cv->dtype, dx));
    if (flags & T2SC_RESIDUAL) T2SC_TRY(upload_as(ctx, residual, n * cv->co, cv->dtype, dr));
    T2SC_TRY(dy.alloc(ctx, n * cv->co * elem_size(cv->dtype)));
    T2SC_TRY(forward_device_impl(cv, c, dx.p, dy.p, flags, dr.p));
    T2SC_TRY(download_as(ctx, dy.p, n * cv->co, cv->dtype, y));
    return check_sync(ctx);
  });
}

}  // extern "C"

// ---------------------------- pipelined chain -----------------------------
//
// A chain over host buffers is bound by the PCIe copies of its input and
// output (f32, both ways), not by the convs. When the rows are ordered by
// (batch, x), as coordinate sets built in lexicographic order are, the rows
// split into contiguous slabs along x; each slab is run on its own rows
// plus a halo as deep as the chain's reach along x, so that its own rows'
// outputs equal the whole set's (a halo row's layer-i result is right while
// its depth is within the reach still left after layer i). Slab uploads,
// slab chains and slab downloads run on three streams, so the upload of
// slab s + 1 and the download of slab s - 1 overlap the convs of slab s and
// each other (host-to-device and device-to-host copies run concurrently).

constexpr int64_t kChainMinRows = 200000;   // smaller sets run unsplit
constexpr int64_t kChainRowsPerSlab = 100000;
constexpr int kChainMaxSlabs = 8;

// Slab plan of a coordinate set for a reach (cached on the set; an empty
// plan means the set runs unsplit: too small, not ordered by (batch, x), or
// halos too large to pay off). Building it reads the coordinates back once.
static int chain_plan(t2sc_coords *c, int64_t reach, const std::vector<t2sc_chain_slab> **out) {
  t2sc_ctx *ctx = c->ctx;
  std::string &err = ctx->last_error;
  auto it = c->chain_plans.find(reach);
  if (it != c->chain_plans.end()) {
    *out = &it->second;
    return T2SC_OK;
  }
  std::vector<t2sc_chain_slab> plan;
  const int64_t n = c->n;
  const int nslab = (int)std::min<int64_t>(kChainMaxSlabs, n / kChainRowsPerSlab);
  if (n >= kChainMinRows && nslab >= 2) {
    std::vector<int32_t> h((size_t)n * 4);
    T2SC_CUDA(cudaMemcpyAsync(h.data(), c->d_coords, (size_t)n * 16, cudaMemcpyDeviceToHost, ctx->stream),
              "chain plan");
    T2SC_CUDA(cudaStreamSynchronize(ctx->stream), "chain plan");
    std::vector<int64_t> key((size_t)n);
    bool sorted = true;
    for (int64_t r = 0; r < n; r++) {
      key[r] = (int64_t)h[4 * r] * (int64_t(1) << 22) + (h[4 * r + 1] + (int64_t(1) << 20));
      if (r > 0 && key[r] < key[r - 1]) {
        sorted = false;
        break;
      }
    }
    if (sorted) {
      // own ranges cut where the (batch, x) key changes, near n * s / nslab
      std::vector<int64_t> cut{0};
      for (int s = 1; s < nslab; s++) {
        int64_t r = std::max(cut.back() + 1, n * s / nslab);
        while (r < n && key[r] == key[r - 1]) r++;
        if (r < n) cut.push_back(r);
      }
      cut.push_back(n);
      int64_t local_max = 0, local_sum = 0;
      for (size_t s = 0; s + 1 < cut.size(); s++) {
        t2sc_chain_slab sl;
        sl.t0 = cut[s];
        sl.t1 = cut[s + 1];
        sl.lo = std::lower_bound(key.begin(), key.end(), key[sl.t0] - reach) - key.begin();
        sl.hi = std::upper_bound(key.begin(), key.end(), key[sl.t1 - 1] + reach) - key.begin();
        local_max = std::max(local_max, sl.hi - sl.lo);
        local_sum += sl.hi - sl.lo;
        plan.push_back(sl);
      }
      // worth it only if the halos stay small next to the own rows
      if (plan.size() < 2 || local_sum > n + n / 3 || local_max > n / 2) plan.clear();
      for (auto &sl : plan) {
        int rc = coords_create_impl(ctx, c->d_coords + 4 * sl.lo, sl.hi - sl.lo, sl.hi - sl.lo, true, &sl.all);
        if (rc == T2SC_OK)
          rc = coords_create_impl(ctx, c->d_coords + 4 * sl.lo, sl.hi - sl.lo, sl.t1 - sl.t0, true, &sl.own,
                                  sl.t0 - sl.lo);
        if (rc != T2SC_OK) {
          for (auto &q : plan) {
            t2sc_coords_destroy(q.all);
            t2sc_coords_destroy(q.own);
          }
          return rc;
        }
      }
    }
  }
  auto ins = c->chain_plans.emplace(reach, std::move(plan));
  *out = &ins.first->second;
  return T2SC_OK;
}

static int chain_pipelined(t2sc_conv *const *convs, int n_layers, t2sc_coords *c,
                           const std::vector<t2sc_chain_slab> &plan, const float *x, float *y, const int *flags,
                           int cmax) {
  t2sc_ctx *ctx = c->ctx;
  std::string &err = ctx->last_error;
  const int dtype = convs[0]->dtype;
  const size_t es = elem_size(dtype);
  const int64_t n = c->n, ci = convs[0]->ci, co = convs[n_layers - 1]->co;
  if (!ctx->up_stream) T2SC_CUDA(cudaStreamCreateWithFlags(&ctx->up_stream, cudaStreamNonBlocking), "chain stream");
  if (!ctx->down_stream)
    T2SC_CUDA(cudaStreamCreateWithFlags(&ctx->down_stream, cudaStreamNonBlocking), "chain stream");
  cudaStream_t cs = ctx->stream, up = ctx->up_stream, dn = ctx->down_stream;
  int64_t local_max = 0;
  for (auto &sl : plan) local_max = std::max(local_max, sl.hi - sl.lo);
  DevBuf din, dout, stage_in, stage_out, b0, b1;
  const bool f32 = dtype == T2SC_DT_F32;
  T2SC_TRY(din.alloc(ctx, n * ci * es));
  T2SC_TRY(dout.alloc(ctx, n * co * es));
  if (!f32) {
    T2SC_TRY(stage_in.alloc(ctx, n * ci * 4));
    T2SC_TRY(stage_out.alloc(ctx, n * co * 4));
  }
  T2SC_TRY(b0.alloc(ctx, local_max * cmax * es));
  T2SC_TRY(b1.alloc(ctx, local_max * cmax * es));
  const size_t ns = plan.size();
  std::vector<cudaEvent_t> ev(2 * ns + 2, nullptr);
  for (auto &e : ev) T2SC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chain event");
  struct EventsGuard {
    std::vector<cudaEvent_t> &v;
    ~EventsGuard() {
      for (auto e : v)
        if (e) cudaEventDestroy(e);
    }
  } guard_ev{ev};
  cudaEvent_t ev_start = ev[2 * ns], ev_end = ev[2 * ns + 1];
  // the copy streams start after the allocations (and earlier work) on the context's stream
  T2SC_CUDA(cudaEventRecord(ev_start, cs), "chain event");
  T2SC_CUDA(cudaStreamWaitEvent(up, ev_start, 0), "chain event");
  T2SC_CUDA(cudaStreamWaitEvent(dn, ev_start, 0), "chain event");
  uint8_t *din8 = (uint8_t *)din.p, *dout8 = (uint8_t *)dout.p;
  // The copy streams carry only copies (back to back, so the copy engines
  // never wait for a conversion kernel); conversions run on the context's
  // stream with the convs.
  int64_t uploaded = 0;
  for (size_t s = 0; s < ns; s++) {
    const t2sc_chain_slab &sl = plan[s];
    // upload: rows [uploaded, hi) (the part of this slab's rows not yet on the device)
    const int64_t r0 = uploaded, r1 = s + 1 == ns ? n : sl.hi;
    if (r1 > r0) {
      const int64_t cnt = (r1 - r0) * ci;
      void *dst = f32 ? (void *)(din8 + r0 * ci * 4) : (void *)((float *)stage_in.p + r0 * ci);
      T2SC_CUDA(cudaMemcpyAsync(dst, x + r0 * ci, cnt * 4, cudaMemcpyHostToDevice, up), "chain upload");
      uploaded = r1;
    }
    T2SC_CUDA(cudaEventRecord(ev[s], up), "chain event");
    // the slab's chain on the context's stream
    T2SC_CUDA(cudaStreamWaitEvent(cs, ev[s], 0), "chain event");
    if (!f32 && r1 > r0)
      T2SC_TRY(f32_to_dtype(ctx, (const float *)stage_in.p + r0 * ci, din8 + r0 * ci * es, (r1 - r0) * ci, dtype));
    const void *cur = din8 + sl.lo * ci * es;
    void *bufs[2] = {b0.p, b1.p};
    for (int i = 0; i < n_layers; i++) {
      const int f = flags ? flags[i] : 0;
      const bool last = i == n_layers - 1;
      t2sc_coords *h = last ? sl.own : sl.all;
      void *outp = last ? (void *)(dout8 + sl.t0 * co * es) : bufs[i & 1];
      const void *res = (f & T2SC_RESIDUAL) ? (const void *)(din8 + (last ? sl.t0 : sl.lo) * ci * es) : nullptr;
      T2SC_TRY(forward_device_impl(convs[i], h, cur, outp, f, res));
      cur = outp;
    }
    const int64_t cnt = (sl.t1 - sl.t0) * co;
    const float *src = f32 ? (const float *)(dout8 + sl.t0 * co * 4) : (const float *)stage_out.p + sl.t0 * co;
    if (!f32) T2SC_TRY(dtype_to_f32(ctx, dout8 + sl.t0 * co * es, (float *)src, cnt, dtype));
    T2SC_CUDA(cudaEventRecord(ev[ns + s], cs), "chain event");
    // download the own rows
    T2SC_CUDA(cudaStreamWaitEvent(dn, ev[ns + s], 0), "chain event");
    T2SC_CUDA(cudaMemcpyAsync(y + sl.t0 * co, src, cnt * 4, cudaMemcpyDeviceToHost, dn), "chain download");
  }
  // the context's stream waits for the last download (buffers are freed on it)
  T2SC_CUDA(cudaEventRecord(ev_end, dn), "chain event");
  T2SC_CUDA(cudaStreamWaitEvent(cs, ev_end, 0), "chain event");
  T2SC_CUDA(cudaEventRecord(ev_end, up), "chain event");
  T2SC_CUDA(cudaStreamWaitEvent(cs, ev_end, 0), "chain event");
  return check_sync(ctx);
}

extern "C" {

int t2sc_conv_chain_forward(t2sc_conv *const *convs, int n_layers, t2sc_coords *c, const float *x, float *y,
                            const int *flags) {
  if (!convs || n_layers <= 0 || !c || !convs[0]) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = convs[0]->ctx;
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    const int dtype = convs[0]->dtype;
    int cmax = convs[0]->ci;
    for (int i = 0; i < n_layers; i++) {
      if (!convs[i] || convs[i]->ctx != ctx || convs[i]->dtype != dtype)
        return fail(ctx, T2SC_ERR_INVALID, "chain: convs must share context and dtype");
      if (i > 0 && convs[i]->ci != convs[i - 1]->co)
        return fail(ctx, T2SC_ERR_INVALID, "chain: Ci of a layer must equal Co of the previous one");
      int f = flags ? flags[i] : 0;
      if ((f & T2SC_RESIDUAL) && convs[i]->co != convs[0]->ci)
        return fail(ctx, T2SC_ERR_INVALID, "chain: residual layer needs Co equal to the chain input width");
      cmax = convs[i]->co > cmax ? convs[i]->co : cmax;
    }
    const int64_t n = c->n;
    if (c->n_targets != n || c->target_begin != 0)
      return fail(ctx, T2SC_ERR_INVALID, "chain: coordinates with halo rows are not chainable");
    if (n == 0) return T2SC_OK;
    if (!x || !y) return fail(ctx, T2SC_ERR_INVALID, "null feature buffer");
    int64_t reach = 0;  // rows a chain output depends on lie within this many x planes
    for (int i = 0; i < n_layers; i++) reach += (int64_t)(convs[i]->kd / 2) * convs[i]->dilation;
    const std::vector<t2sc_chain_slab> *plan = nullptr;
    T2SC_TRY(chain_plan(c, reach, &plan));
    if (!plan->empty()) return chain_pipelined(convs, n_layers, c, *plan, x, y, flags, cmax);
    DevBuf din, b0, b1;
    T2SC_TRY(upload_as(ctx, x, n * convs[0]->ci, dtype, din));
    T2SC_TRY(b0.alloc(ctx, n * cmax * elem_size(dtype)));
    T2SC_TRY(b1.alloc(ctx, n * cmax * elem_size(dtype)));
    const void *cur = din.p;
    void *bufs[2] = {b0.p, b1.p};
    for (int i = 0; i < n_layers; i++) {
      int f = flags ? flags[i] : 0;
      void *out = bufs[i & 1];
      T2SC_TRY(forward_device_impl(convs[i], c, cur, out, f, (f & T2SC_RESIDUAL) ? din.p : nullptr));
      cur = out;
    }
    T2SC_TRY(download_as(ctx, cur, n * convs[n_layers - 1]->co, dtype, y));
    return check_sync(ctx);
  });
}

// ------------------------------- subdivision -------------------------------

static int sub_args_ok(t2sc_ctx *ctx, int64_t n, const int32_t *coords, const float *sub, int keep_mode,
                       const void *feats, int c, int feats_mode, const int32_t *out_coords, const void *out_feats,
                       const int64_t *m) {
  if (!m) return fail(ctx, T2SC_ERR_INVALID, "subdivide: null m");
  if (n < 0 || (n > 0 && (!coords || !sub || !out_coords))) return fail(ctx, T2SC_ERR_INVALID, "subdivide: null input");
  if (n >= (int64_t(1) << 28)) return fail(ctx, T2SC_ERR_UNSUPPORTED, "subdivide: more than 2^28 parents");
  if (keep_mode != T2SC_SUB_NONZERO && keep_mode != T2SC_SUB_POSITIVE)
    return fail(ctx, T2SC_ERR_INVALID, "subdivide: unknown keep mode");
  if (feats_mode != T2SC_FEATS_NONE && feats_mode != T2SC_FEATS_UPSAMPLE && feats_mode != T2SC_FEATS_C2S)
    return fail(ctx, T2SC_ERR_INVALID, "subdivide: unknown feature mode");
  if (feats_mode != T2SC_FEATS_NONE && n > 0 && (!feats || !out_feats || c <= 0))
    return fail(ctx, T2SC_ERR_INVALID, "subdivide: feature buffers and C > 0 required");
  return T2SC_OK;
}

int t2sc_subdivide_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub, int keep_mode,
                          const void *feats, int c, int feats_mode, int dtype, int32_t *out_coords, void *out_feats,
                          int32_t *out_parent, int32_t *out_subidx, int64_t *m) {
  if (!ctx) return T2SC_ERR_INVALID;
  T2SC_TRY(sub_args_ok(ctx, n, coords, sub, keep_mode, feats, c, feats_mode, out_coords, out_feats, m));
  if (dtype != T2SC_DT_F32 && dtype != T2SC_DT_F16 && dtype != T2SC_DT_BF16)
    return fail(ctx, T2SC_ERR_INVALID, "subdivide: unknown dtype");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    return subdivide_device(ctx, coords, n, sub, keep_mode, feats, c, feats_mode, dtype, out_coords, out_feats,
                            out_parent, out_subidx, m, ctx->last_error);
  });
}

int t2sc_fdg_head_device(t2sc_ctx *ctx, const float *feats, int64_t t, double margin, float *vertices,
                         float *intersected, float *quad_lerp) {
  if (!ctx) return T2SC_ERR_INVALID;
  if (t < 0) return fail(ctx, T2SC_ERR_INVALID, "fdg_head: t < 0");
  if (t > 0 && (!feats || !vertices || !intersected || !quad_lerp))
    return fail(ctx, T2SC_ERR_INVALID, "fdg_head: null buffer");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    return fdg_head_device(ctx, feats, t, (float)margin, vertices, intersected, quad_lerp, ctx->last_error);
  });
}

int t2sc_cascade_coords_device(t2sc_ctx *ctx, const int32_t *hr_coords, int64_t n, int lr_resolution,
                               int resolution, int64_t max_num_tokens, int32_t *out_coords,
                               int64_t *num_tokens, int *hr_resolution) {
  if (!ctx) return T2SC_ERR_INVALID;
  if (!num_tokens || !hr_resolution) return fail(ctx, T2SC_ERR_INVALID, "cascade_coords: null result pointer");
  if (n < 0 || n >= (int64_t(1) << 31)) return fail(ctx, T2SC_ERR_INVALID, "cascade_coords: need 0 <= n < 2^31");
  if (n > 0 && (!hr_coords || !out_coords)) return fail(ctx, T2SC_ERR_INVALID, "cascade_coords: null coordinates");
  if (lr_resolution <= 0 || resolution <= 0 || resolution > (1 << 24))
    return fail(ctx, T2SC_ERR_INVALID, "cascade_coords: need lr_resolution > 0 and 0 < resolution <= 2^24");
  if (max_num_tokens <= 0) return fail(ctx, T2SC_ERR_INVALID, "cascade_coords: max_num_tokens must be > 0");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    return cascade_coords_device(ctx, hr_coords, n, lr_resolution, resolution, max_num_tokens, out_coords,
                                 num_tokens, hr_resolution, ctx->last_error);
  });
}

int t2sc_grid_sample_trilinear_device(t2sc_coords *coords, const float *feats, int c, int grid_size,
                                      const float *query, int64_t l, float *out) {
  if (!coords) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = coords->ctx;
  if (c < 1 || l < 0) return fail(ctx, T2SC_ERR_INVALID, "grid_sample: need c >= 1 and l >= 0");
  if (grid_size < 1 || grid_size > 1536)
    return fail(ctx, T2SC_ERR_UNSUPPORTED, "grid_sample: grid_size must be in [1, 1536]");
  if (l > 0 && (!query || !out || (coords->n > 0 && !feats)))
    return fail(ctx, T2SC_ERR_INVALID, "grid_sample: null buffer");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    return grid_sample_device(coords, feats, c, grid_size, query, l, out, ctx->last_error);
  });
}

int t2sc_layernorm_device(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w,
                          const float *b, float eps, int flags, int dtype) {
  if (!ctx) return T2SC_ERR_INVALID;
  if (rows < 0 || c < 1 || c > 1024) return fail(ctx, T2SC_ERR_INVALID, "layernorm: need rows >= 0, 1 <= c <= 1024");
  if (rows > 0 && (!x || !y)) return fail(ctx, T2SC_ERR_INVALID, "layernorm: null feature buffer");
  if ((w == nullptr) != (b == nullptr)) return fail(ctx, T2SC_ERR_INVALID, "layernorm: w and b must both be set or both NULL");
  if (!(eps >= 0.f)) return fail(ctx, T2SC_ERR_INVALID, "layernorm: eps must be >= 0");
  if (flags & ~T2SC_SILU) return fail(ctx, T2SC_ERR_INVALID, "layernorm: only T2SC_SILU is a valid flag");
  if (dtype != T2SC_DT_F32 && dtype != T2SC_DT_F16 && dtype != T2SC_DT_BF16)
    return fail(ctx, T2SC_ERR_INVALID, "layernorm: unknown dtype");
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    return layernorm_device(ctx, x, y, rows, c, w, b, eps, flags, dtype, ctx->last_error);
  });
}

int t2sc_subdivide(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub, int keep_mode,
                   const float *feats, int c, int feats_mode, int32_t *out_coords, float *out_feats,
                   int64_t *out_parent, int64_t *out_subidx, int64_t *m) {
  if (!ctx) return T2SC_ERR_INVALID;
  T2SC_TRY(sub_args_ok(ctx, n, coords, sub, keep_mode, feats, c, feats_mode, out_coords, out_feats, m));
  return guarded(ctx, [&]() -> int {
    DeviceGuard g(ctx->device);
    std::string &err = ctx->last_error;
    *m = 0;
    if (n == 0) return T2SC_OK;
    const int64_t fin = feats_mode == T2SC_FEATS_C2S ? 8 * (int64_t)c : c;
    DevBuf dc, ds, dfi, dco, dfo, dpar, dsub;
    T2SC_TRY(dc.alloc(ctx, n * 16));
    T2SC_TRY(ds.alloc(ctx, n * 32));
    T2SC_TRY(dco.alloc(ctx, 8 * n * 16));
    T2SC_TRY(dpar.alloc(ctx, 8 * n * 4));
    T2SC_TRY(dsub.alloc(ctx, 8 * n * 4));
    T2SC_CUDA(cudaMemcpyAsync(dc.p, coords, n * 16, cudaMemcpyHostToDevice, ctx->stream), "subdivide upload");
    T2SC_CUDA(cudaMemcpyAsync(ds.p, sub, n * 32, cudaMemcpyHostToDevice, ctx->stream), "subdivide upload");
    if (feats_mode != T2SC_FEATS_NONE) {
      T2SC_TRY(dfi.alloc(ctx, n * fin * 4));
      T2SC_TRY(dfo.alloc(ctx, 8 * n * (int64_t)c * 4));
      T2SC_CUDA(cudaMemcpyAsync(dfi.p, feats, n * fin * 4, cudaMemcpyHostToDevice, ctx->stream), "subdivide upload");
    }
    int64_t mm = 0;
    T2SC_TRY(subdivide_device(ctx, (const int32_t *)dc.p, n, (const float *)ds.p, keep_mode, dfi.p, c, feats_mode,
                              T2SC_DT_F32, (int32_t *)dco.p, dfo.p, (int32_t *)dpar.p, (int32_t *)dsub.p, &mm, err));
    std::vector<int32_t> par(out_parent ? mm : 0), sid(out_subidx ? mm : 0);
    if (mm > 0) {
      T2SC_CUDA(cudaMemcpyAsync(out_coords, dco.p, mm * 16, cudaMemcpyDeviceToHost, ctx->stream), "subdivide dl");
      if (feats_mode != T2SC_FEATS_NONE)
        T2SC_CUDA(cudaMemcpyAsync(out_feats, dfo.p, mm * (int64_t)c * 4, cudaMemcpyDeviceToHost, ctx->stream),
                  "subdivide dl");
      if (out_parent)
        T2SC_CUDA(cudaMemcpyAsync(par.data(), dpar.p, mm * 4, cudaMemcpyDeviceToHost, ctx->stream), "subdivide dl");
      if (out_subidx)
        T2SC_CUDA(cudaMemcpyAsync(sid.data(), dsub.p, mm * 4, cudaMemcpyDeviceToHost, ctx->stream), "subdivide dl");
    }
    T2SC_TRY(check_sync(ctx));
    for (int64_t e = 0; e < (int64_t)par.size(); e++) out_parent[e] = par[e];
    for (int64_t e = 0; e < (int64_t)sid.size(); e++) out_subidx[e] = sid[e];
    *m = mm;
    return T2SC_OK;
  });
}

}  // extern "C"
