// 2x subdivision: child-coordinate generation and mask compaction.
// Reference: SparseUpsample.forward_subdivision
// (trellis2_mojo/sparse/spatial/basic.mojo:144-174) and
// SparseChannel2Spatial.forward_subdivision/_unfold
// (trellis2_mojo/sparse/spatial/spatial2channel.mojo:97-145): children are
// emitted parent-major with the child index c ascending, and child c of
// (b,x,y,z) is (b, 2x + (c&1), 2y + ((c>>1)&1), 2z + ((c>>2)&1)).
//
// Three passes: (1) per parent, the 8-bit keep mask and its popcount;
// (2) an exclusive shuffle-scan of the counts (scan.cu) gives each parent's
// first output row; (3) eight lanes per parent write its children and their
// feature rows (16-byte vectors when the row size allows). The child count
// is read back once, at the end.
#include <mutex>

#include "internal.h"

namespace t2sc {
namespace {

__global__ void sub_count_kernel(const float *__restrict__ sub, int64_t n, int positive, uint8_t *__restrict__ masks,
                                 int32_t *__restrict__ counts) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const float4 *s4 = reinterpret_cast<const float4 *>(sub + r * 8);
  float4 a = s4[0], b = s4[1];
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t m = 0;
#pragma unroll
  for (int c = 0; c < 8; c++) m |= (positive ? (v[c] > 0.0f) : (v[c] != 0.0f)) ? (1u << c) : 0u;
  masks[r] = (uint8_t)m;
  counts[r] = __popc(m);
}

// Eight lanes per parent (four parents per warp): lane c handles child slot
// c; a kept child lands at row offs[r] + popcount(mask & ((1 << c) - 1)), so
// children stay parent-major with c ascending. Each kept lane writes its
// coordinates, parent / slot entries and its feature row (vpr vectors).
// parent / subidx / in may be null (nothing written or copied for them).
template <typename V>
__global__ void __launch_bounds__(256) sub_children_kernel(const int4 *__restrict__ coords,
                                                           const uint8_t *__restrict__ masks,
                                                           const int64_t *__restrict__ offs, int64_t n,
                                                           const V *__restrict__ in, V *__restrict__ out, int vpr,
                                                           int c2s, int4 *__restrict__ out_coords,
                                                           int32_t *__restrict__ parent, int32_t *__restrict__ subidx) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r = t >> 3;
  const int c = (int)(t & 7);
  if (r >= n) return;
  const uint32_t m = masks[r];
  if (!((m >> c) & 1u)) return;
  const int64_t e = offs[r] + __popc(m & ((1u << c) - 1u));
  const int4 p = coords[r];
  out_coords[e] = make_int4(p.x, p.y * 2 + (c & 1), p.z * 2 + ((c >> 1) & 1), p.w * 2 + ((c >> 2) & 1));
  if (parent) parent[e] = (int32_t)r;
  if (subidx) subidx[e] = c;
  if (!in) return;
  const V *src = in + (c2s ? (r * 8 + c) : r) * vpr;
  V *dst = out + e * vpr;
  for (int v = 0; v < vpr; v++) dst[v] = src[v];
}

inline unsigned nblk(int64_t n) { return (unsigned)((n + 255) / 256); }

// Children, parent / slot entries and feature rows of every kept child, in
// one launch (no host read of the child count needed first).
int emit_children(t2sc_ctx *ctx, const int32_t *coords, const uint8_t *masks, const int64_t *offs, int64_t n,
                  const void *feats, int c, int feats_mode, int dtype, int32_t *out_coords, void *out_feats,
                  int32_t *par, int32_t *sidx, std::string &err) {
  cudaStream_t st = ctx->stream;
  const bool copy = feats_mode != T2SC_FEATS_NONE;
  const int64_t row_bytes = copy ? (int64_t)c * (dtype == T2SC_DT_F32 ? 4 : 2) : 16;
  const int c2s = feats_mode == T2SC_FEATS_C2S;
  const unsigned grid = (unsigned)((n * 8 + 255) / 256);
  if (row_bytes % 16 == 0) {
    sub_children_kernel<uint4><<<grid, 256, 0, st>>>((const int4 *)coords, masks, offs, n,
                                                     copy ? (const uint4 *)feats : nullptr, (uint4 *)out_feats,
                                                     (int)(row_bytes / 16), c2s, (int4 *)out_coords, par, sidx);
  } else if (row_bytes % 4 == 0) {
    sub_children_kernel<uint32_t><<<grid, 256, 0, st>>>((const int4 *)coords, masks, offs, n,
                                                        (const uint32_t *)feats, (uint32_t *)out_feats,
                                                        (int)(row_bytes / 4), c2s, (int4 *)out_coords, par, sidx);
  } else {
    sub_children_kernel<uint16_t><<<grid, 256, 0, st>>>((const int4 *)coords, masks, offs, n,
                                                        (const uint16_t *)feats, (uint16_t *)out_feats,
                                                        (int)(row_bytes / 2), c2s, (int4 *)out_coords, par, sidx);
  }
  T2SC_LAUNCHED(ctx, "sub_children");
  return T2SC_OK;
}
}  // namespace

int subdivide_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub, int keep_mode,
                     const void *feats, int c, int feats_mode, int dtype, int32_t *out_coords, void *out_feats,
                     int32_t *out_parent, int32_t *out_subidx, int64_t *m_out, std::string &err) {
  cudaStream_t st = ctx->stream;
  *m_out = 0;
  if (n == 0) return T2SC_OK;
  uint8_t *masks = nullptr;
  int32_t *counts = nullptr, *par = out_parent, *sidx = out_subidx;
  int64_t *offs = nullptr;
  T2SC_CUDA(cudaMallocAsync((void **)&masks, n, st), "subdiv scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&counts, n * sizeof(int32_t), st), "subdiv scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&offs, (n + 1) * sizeof(int64_t), st), "subdiv scratch");
  sub_count_kernel<<<nblk(n), 256, 0, st>>>(sub, n, keep_mode == T2SC_SUB_POSITIVE, masks, counts);
  T2SC_LAUNCHED(ctx, "sub_count");
  int rc = scan_counts(ctx, counts, n, offs, offs + n);
  if (rc != T2SC_OK) return rc;
  rc = emit_children(ctx, coords, masks, offs, n, feats, c, feats_mode, dtype, out_coords, out_feats, par, sidx, err);
  if (rc != T2SC_OK) return rc;
  int64_t m = 0;
  T2SC_CUDA(cudaMemcpyAsync(&m, offs + n, sizeof(int64_t), cudaMemcpyDeviceToHost, st), "subdiv count");
  T2SC_CUDA(cudaStreamSynchronize(st), "subdiv count");
  cudaFreeAsync(masks, st);
  cudaFreeAsync(counts, st);
  cudaFreeAsync(offs, st);
  *m_out = m;
  return T2SC_OK;
}

}  // namespace t2sc

// ---------------------------------------------------------------------------
// Allocation-free subdivision (t2sc_subdivide_noalloc_device).
//
// Some callers cannot allocate device memory while they run this step: a
// host runtime that hands the library a fixed memory budget up front, or an
// engine that must not touch the CUDA allocator (and its implicit
// synchronisation) in the middle of a decode pass. For them the scratch of
// the subdivision (keep masks, per-parent counts and offsets, and the scan's
// block sums) lives in one file-scope device array instead of stream-ordered
// allocations. Its size is fixed at build time for up to
// kNoAllocMaxParents parents; every GPU that loads the library holds it
// until the process exits.
namespace t2sc {
namespace {

constexpr int64_t kNoAllocMaxParents = int64_t(1) << 20;
constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t kNaMasks = 0;
constexpr size_t kNaCounts = align256(kNaMasks + kNoAllocMaxParents);
constexpr size_t kNaOffs = align256(kNaCounts + 4 * kNoAllocMaxParents);
constexpr size_t kNaBlocks = align256(kNaOffs + 8 * (kNoAllocMaxParents + 1));
constexpr size_t kNaBytes =
    align256(kNaBlocks + 8 * ((kNoAllocMaxParents + kScanTileItems - 1) / kScanTileItems));

// Shared by every call on a device; the last call's contents stay in it.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNaBytes];

// Device address of g_noalloc_scratch per device, looked up once with that
// device current (in host code the symbol is only a host-side handle).
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[128] = {};

int noalloc_scratch(int device, uint8_t **out, std::string &err) {
  if (device < 0 || device >= 128) {
    err = "device ordinal out of range";
    return T2SC_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      err = std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e);
      return T2SC_ERR_CUDA;
    }
    g_noalloc_ptr[device] = static_cast<uint8_t *>(p);
  }
  *out = g_noalloc_ptr[device];
  return T2SC_OK;
}

}  // namespace
}  // namespace t2sc

extern "C" int t2sc_subdivide_noalloc_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub,
                                             int keep_mode, const void *feats, int c, int feats_mode, int dtype,
                                             int32_t *out_coords, void *out_feats, int32_t *out_parent,
                                             int32_t *out_subidx, int64_t *m) {
  using namespace t2sc;
  if (!ctx) return T2SC_ERR_INVALID;
  std::string &err = ctx->last_error;
  if (!m) {
    err = "subdivide_noalloc: null m";
    return T2SC_ERR_INVALID;
  }
  *m = 0;
  if (n < 0 || n > kNoAllocMaxParents) {
    err = "subdivide_noalloc: n = " + std::to_string(n) + " parents is outside the static scratch limit of " +
          std::to_string(kNoAllocMaxParents) + "; use t2sc_subdivide_device";
    return T2SC_ERR_INVALID;
  }
  if (keep_mode != T2SC_SUB_NONZERO && keep_mode != T2SC_SUB_POSITIVE) {
    err = "subdivide_noalloc: unknown keep mode";
    return T2SC_ERR_INVALID;
  }
  if (feats_mode != T2SC_FEATS_NONE && feats_mode != T2SC_FEATS_UPSAMPLE && feats_mode != T2SC_FEATS_C2S) {
    err = "subdivide_noalloc: unknown feature mode";
    return T2SC_ERR_INVALID;
  }
  if (dtype != T2SC_DT_F32 && dtype != T2SC_DT_F16 && dtype != T2SC_DT_BF16) {
    err = "subdivide_noalloc: unknown dtype";
    return T2SC_ERR_INVALID;
  }
  if (n == 0) return T2SC_OK;
  if (!coords || !sub || !out_coords || !out_parent || !out_subidx ||
      (feats_mode != T2SC_FEATS_NONE && (!feats || !out_feats || c <= 0))) {
    err = "subdivide_noalloc: null buffer (out_parent and out_subidx are required here)";
    return T2SC_ERR_INVALID;
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  int rc = [&]() -> int {
    uint8_t *scr = nullptr;
    int r = noalloc_scratch(ctx->device, &scr, err);
    if (r != T2SC_OK) return r;
    uint8_t *masks = scr + kNaMasks;
    int32_t *counts = reinterpret_cast<int32_t *>(scr + kNaCounts);
    int64_t *offs = reinterpret_cast<int64_t *>(scr + kNaOffs);
    int64_t *blocks = reinterpret_cast<int64_t *>(scr + kNaBlocks);
    cudaStream_t st = ctx->stream;
    // every scratch word read below is first written by this call (masks and
    // counts for all n parents, offsets and block sums by the scan), so
    // nothing has to be cleared
    sub_count_kernel<<<nblk(n), 256, 0, st>>>(sub, n, keep_mode == T2SC_SUB_POSITIVE, masks, counts);
    T2SC_LAUNCHED(ctx, "sub_count");
    r = scan_counts_into(ctx, counts, n, offs, offs + n, blocks);
    if (r != T2SC_OK) return r;
    r = emit_children(ctx, coords, masks, offs, n, feats, c, feats_mode, dtype, out_coords, out_feats, out_parent,
                      out_subidx, err);
    if (r != T2SC_OK) return r;
    int64_t mm = 0;
    T2SC_CUDA(cudaMemcpyAsync(&mm, offs + n, sizeof(int64_t), cudaMemcpyDeviceToHost, st), "subdivide count");
    T2SC_CUDA(cudaStreamSynchronize(st), "subdivide count");
    *m = mm;
    return T2SC_OK;
  }();
  int cur = -1;
  if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  return rc;
}
