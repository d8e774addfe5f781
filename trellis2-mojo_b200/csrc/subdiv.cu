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
// first output row; (3) children and their feature rows are written, the
// features as 16-byte vectors when the row size allows.
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

__global__ void sub_emit_kernel(const int4 *__restrict__ coords, const uint8_t *__restrict__ masks,
                                const int64_t *__restrict__ offs, int64_t n, int4 *__restrict__ out_coords,
                                int32_t *__restrict__ parent, int32_t *__restrict__ subidx) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  uint32_t m = masks[r];
  if (!m) return;
  int4 p = coords[r];
  int64_t e = offs[r];
  while (m) {
    int c = __ffs(m) - 1;
    m &= m - 1;
    out_coords[e] = make_int4(p.x, p.y * 2 + (c & 1), p.z * 2 + ((c >> 1) & 1), p.w * 2 + ((c >> 2) & 1));
    parent[e] = (int32_t)r;
    subidx[e] = c;
    e++;
  }
}

// out[e, :] = in[parent[e], slot*C : slot*C + C] with slot = subidx[e] (C2S) or 0.
template <typename V>
__global__ void sub_feats_kernel(const V *__restrict__ in, V *__restrict__ out, const int32_t *__restrict__ parent,
                                 const int32_t *__restrict__ subidx, int64_t m, int vec_per_row, int c2s) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * vec_per_row) return;
  int64_t e = i / vec_per_row;
  int v = (int)(i % vec_per_row);
  int64_t p = parent[e];
  int64_t src = c2s ? (p * 8 + subidx[e]) * vec_per_row + v : p * vec_per_row + v;
  out[i] = in[src];
}

inline unsigned nblk(int64_t n) { return (unsigned)((n + 255) / 256); }
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
  if (!par) T2SC_CUDA(cudaMallocAsync((void **)&par, 8 * n * sizeof(int32_t), st), "subdiv scratch");
  if (!sidx) T2SC_CUDA(cudaMallocAsync((void **)&sidx, 8 * n * sizeof(int32_t), st), "subdiv scratch");
  sub_count_kernel<<<nblk(n), 256, 0, st>>>(sub, n, keep_mode == T2SC_SUB_POSITIVE, masks, counts);
  T2SC_LAUNCHED(ctx, "sub_count");
  int rc = scan_counts(ctx, counts, n, offs, offs + n);
  if (rc != T2SC_OK) return rc;
  sub_emit_kernel<<<nblk(n), 256, 0, st>>>((const int4 *)coords, masks, offs, n, (int4 *)out_coords, par, sidx);
  T2SC_LAUNCHED(ctx, "sub_emit");
  int64_t m = 0;
  T2SC_CUDA(cudaMemcpyAsync(&m, offs + n, sizeof(int64_t), cudaMemcpyDeviceToHost, st), "subdiv count");
  T2SC_CUDA(cudaStreamSynchronize(st), "subdiv count");
  if (feats_mode != T2SC_FEATS_NONE && m > 0) {
    const int64_t row_bytes = (int64_t)c * (dtype == T2SC_DT_F32 ? 4 : 2);
    const int c2s = feats_mode == T2SC_FEATS_C2S;
    if (row_bytes % 16 == 0) {
      int vpr = (int)(row_bytes / 16);
      sub_feats_kernel<uint4><<<nblk(m * vpr), 256, 0, st>>>((const uint4 *)feats, (uint4 *)out_feats, par, sidx, m,
                                                            vpr, c2s);
    } else if (row_bytes % 4 == 0) {
      int vpr = (int)(row_bytes / 4);
      sub_feats_kernel<uint32_t><<<nblk(m * vpr), 256, 0, st>>>((const uint32_t *)feats, (uint32_t *)out_feats, par,
                                                               sidx, m, vpr, c2s);
    } else {
      int vpr = (int)(row_bytes / 2);
      sub_feats_kernel<uint16_t><<<nblk(m * vpr), 256, 0, st>>>((const uint16_t *)feats, (uint16_t *)out_feats, par,
                                                               sidx, m, vpr, c2s);
    }
    T2SC_LAUNCHED(ctx, "sub_feats");
  }
  cudaFreeAsync(masks, st);
  cudaFreeAsync(counts, st);
  cudaFreeAsync(offs, st);
  if (par != out_parent) cudaFreeAsync(par, st);
  if (sidx != out_subidx) cudaFreeAsync(sidx, st);
  *m_out = m;
  return T2SC_OK;
}

}  // namespace t2sc
