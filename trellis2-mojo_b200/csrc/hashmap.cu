// Coordinate hash, 27-offset neighbour map and its exports.
//
// Reference semantics (trellis2_mojo/sparse/conv.mojo:56-96):
//  * key = ((b*2048 + x + 512)*2048 + y + 512)*2048 + z + 512, the same
//    int64 arithmetic for stored rows and for probes (so an out-of-range
//    probe aliases exactly as it does in the reference);
//  * the dictionary keeps the LAST row inserted for a key (Dict overwrite),
//    reproduced here with atomicMax on the row index;
//  * offset k = kz*Kh*Kw + ky*Kw + kx moves columns 1, 2, 3 by
//    (kz - Kd/2, ky - Kh/2, kx - Kw/2) * dilation.
//
// Device layout: open-addressing table of int64 keys / int32 rows at load
// factor <= 0.5; nbr[k][r] (k-major, -1 = miss) so that one offset of a
// 128-row tile is one contiguous 512-byte read; a 32-bit occupancy mask per
// row. For the conv, rows are stably radix-sorted by that mask so that rows
// with the same neighbour pattern share a tile and a tile only visits the
// offsets some of its rows use.
#include <cub/device/device_radix_sort.cuh>

#include "internal.h"

namespace t2sc {
namespace {

constexpr int64_t kEmpty = -1;

__device__ __forceinline__ int64_t pack_key(int64_t b, int64_t x, int64_t y, int64_t z) {
  return ((b * 2048 + x + 512) * 2048 + y + 512) * 2048 + z + 512;
}

__device__ __forceinline__ uint64_t mix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdULL;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ULL;
  k ^= k >> 33;
  return k;
}

__global__ void hash_insert_kernel(const int4 *__restrict__ coords, int64_t n, unsigned long long *keys,
                                   int32_t *vals, uint64_t hmask, int *err) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  int4 c = coords[r];
  if (c.x < 0 || c.y < -512 || c.y >= 1536 || c.z < -512 || c.z >= 1536 || c.w < -512 || c.w >= 1536) {
    atomicOr(err, kDevErrRange);
    return;
  }
  unsigned long long key = (unsigned long long)pack_key(c.x, c.y, c.z, c.w);
  uint64_t s = mix64(key) & hmask;
  for (uint64_t probe = 0; probe <= hmask; probe++) {
    unsigned long long prev = atomicCAS(&keys[s], (unsigned long long)kEmpty, key);
    if (prev == (unsigned long long)kEmpty || prev == key) {
      atomicMax(&vals[s], (int32_t)r);  // the last row with this key wins
      return;
    }
    s = (s + 1) & hmask;
  }
  atomicOr(err, kDevErrHashFull);
}

__device__ __forceinline__ int32_t hash_find(const int64_t *__restrict__ keys, const int32_t *__restrict__ vals,
                                             uint64_t hmask, int64_t key) {
  if (key == kEmpty) return -1;
  uint64_t s = mix64((uint64_t)key) & hmask;
  for (uint64_t probe = 0; probe <= hmask; probe++) {
    int64_t k = keys[s];
    if (k == key) return vals[s];
    if (k == kEmpty) return -1;
    s = (s + 1) & hmask;
  }
  return -1;
}

__global__ void neighbor_map_kernel(const int4 *__restrict__ coords, int64_t n, const int64_t *__restrict__ keys,
                                    const int32_t *__restrict__ vals, uint64_t hmask, int kd, int kh, int kw,
                                    int dil, int32_t *__restrict__ nbr, uint32_t *__restrict__ mask,
                                    unsigned long long *__restrict__ n_edges) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t m = 0;
  if (r < n) {
    int4 c = coords[r];
    int k = 0;
    for (int kz = 0; kz < kd; kz++)
      for (int ky = 0; ky < kh; ky++)
        for (int kx = 0; kx < kw; kx++, k++) {
          int64_t key = pack_key(c.x, (int64_t)c.y + (int64_t)(kz - kd / 2) * dil,
                                 (int64_t)c.z + (int64_t)(ky - kh / 2) * dil,
                                 (int64_t)c.w + (int64_t)(kx - kw / 2) * dil);
          int32_t hit = hash_find(keys, vals, hmask, key);
          nbr[(int64_t)k * n + r] = hit;
          m |= (hit >= 0 ? 1u : 0u) << k;
        }
    mask[r] = m;
  }
  // warp-aggregated edge count
  unsigned cnt = __popc(m);
  for (int d = 16; d > 0; d >>= 1) cnt += __shfl_down_sync(0xffffffffu, cnt, d);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(n_edges, (unsigned long long)cnt);
}

__global__ void iota_kernel(int32_t *v, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = (int32_t)i;
}

// One 128-thread block per tile: permuted neighbour rows + tile offset mask.
__global__ void __launch_bounds__(kTileRows) sorted_tiles_kernel(const int32_t *__restrict__ nbr,
                                                                const uint32_t *__restrict__ mask,
                                                                const int32_t *__restrict__ perm_in, int64_t n,
                                                                int64_t n_pad, int kvol,
                                                                int32_t *__restrict__ perm_out,
                                                                int32_t *__restrict__ nbr_sorted,
                                                                uint32_t *__restrict__ tile_mask) {
  __shared__ uint32_t wm[kTileRows / 32];
  int64_t p = (int64_t)blockIdx.x * kTileRows + threadIdx.x;
  int32_t row = p < n ? perm_in[p] : -1;
  perm_out[p] = row;
  uint32_t m = row >= 0 ? mask[row] : 0u;
  for (int k = 0; k < kvol; k++) nbr_sorted[(int64_t)k * n_pad + p] = row >= 0 ? nbr[(int64_t)k * n + row] : -1;
  m = __reduce_or_sync(0xffffffffu, m);
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int i = 0; i < kTileRows / 32; i++) t |= wm[i];
    tile_mask[blockIdx.x] = t;
  }
}

__global__ void edge_flags_kernel(const int32_t *__restrict__ nbr, int64_t total, int32_t *__restrict__ flags) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) flags[i] = nbr[i] >= 0 ? 1 : 0;
}

__global__ void edge_emit_kernel(const int32_t *__restrict__ nbr, int64_t n, int64_t total,
                                 const int64_t *__restrict__ pos, int64_t *__restrict__ src,
                                 int64_t *__restrict__ tgt, int64_t *__restrict__ kidx) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int32_t s = nbr[i];
  if (s < 0) return;
  int64_t p = pos[i];
  src[p] = s;
  tgt[p] = i % n;
  kidx[p] = i / n;
}

__global__ void row_counts_kernel(const uint32_t *__restrict__ mask, int64_t n, int32_t *__restrict__ cnt) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) cnt[r] = __popc(mask[r]);
}

__global__ void csr_emit_kernel(const int32_t *__restrict__ nbr, const uint32_t *__restrict__ mask, int64_t n,
                                const int64_t *__restrict__ row_start, int64_t *__restrict__ src_s,
                                int64_t *__restrict__ kidx_s) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  uint32_t m = mask[r];
  int64_t p = row_start[r];
  while (m) {
    int k = __ffs(m) - 1;
    m &= m - 1;
    src_s[p] = nbr[(int64_t)k * n + r];
    kidx_s[p] = k;
    p++;
  }
}

inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

int build_hash(t2sc_coords *c, std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  uint64_t cap = 1024;
  while (cap < (uint64_t)(2 * c->n)) cap <<= 1;
  c->hcap = cap;
  T2SC_CUDA(cudaMallocAsync((void **)&c->d_keys, cap * sizeof(int64_t), ctx->stream), "hash keys");
  T2SC_CUDA(cudaMallocAsync((void **)&c->d_vals, cap * sizeof(int32_t), ctx->stream), "hash vals");
  T2SC_CUDA(cudaMemsetAsync(c->d_keys, 0xff, cap * sizeof(int64_t), ctx->stream), "hash init");
  T2SC_CUDA(cudaMemsetAsync(c->d_vals, 0xff, cap * sizeof(int32_t), ctx->stream), "hash init");
  if (c->n > 0) {
    hash_insert_kernel<<<nblk(c->n, 256), 256, 0, ctx->stream>>>((const int4 *)c->d_coords, c->n,
                                                               (unsigned long long *)c->d_keys, c->d_vals,
                                                               cap - 1, ctx->d_err);
    T2SC_LAUNCHED(ctx, "hash_insert");
  }
  int flags = 0;
  int rc = read_dev_err(ctx, &flags);
  if (rc != T2SC_OK) return rc;
  if (flags & kDevErrRange) {
    err = "coordinates outside the packable range: need batch >= 0 and x, y, z in [-512, 1536)";
    return T2SC_ERR_RANGE;
  }
  if (flags & kDevErrHashFull) {
    err = "coordinate hash full";
    return T2SC_ERR_INVALID;
  }
  return T2SC_OK;
}

void free_map(t2sc_map *m) {
  if (!m) return;
  cudaFree(m->nbr);
  cudaFree(m->mask);
  cudaFree(m->perm);
  cudaFree(m->nbr_sorted);
  cudaFree(m->tile_mask);
  delete m;
}

__global__ void identity_map_kernel(int64_t n, int64_t n_pad, int32_t *__restrict__ nbr, uint32_t *__restrict__ mask,
                                    int32_t *__restrict__ perm, int32_t *__restrict__ nbr_sorted,
                                    uint32_t *__restrict__ tile_mask) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_pad) return;
  const int32_t r = p < n ? (int32_t)p : -1;
  perm[p] = r;
  nbr_sorted[p] = r;
  if (p < n) nbr[p] = r, mask[p] = 1u;
  if (p % kTileRows == 0) tile_mask[p / kTileRows] = 1u;  // every tile holds >= 1 row
}

int build_identity_map(t2sc_ctx *ctx, int64_t n, t2sc_map **out, std::string &err) {
  std::unique_ptr<t2sc_map, void (*)(t2sc_map *)> m(new t2sc_map(), free_map);
  m->kvol = 1;
  m->n = m->n_src = m->n_edges = n;
  m->ntiles = (n + kTileRows - 1) / kTileRows;
  m->n_pad = m->ntiles * kTileRows;
  const size_t np = (size_t)(m->n_pad > 0 ? m->n_pad : 1), nn = (size_t)(n > 0 ? n : 1);
  T2SC_CUDA(cudaMalloc((void **)&m->nbr, sizeof(int32_t) * nn), "identity map");
  T2SC_CUDA(cudaMalloc((void **)&m->mask, sizeof(uint32_t) * nn), "identity map");
  T2SC_CUDA(cudaMalloc((void **)&m->perm, sizeof(int32_t) * np), "identity map");
  T2SC_CUDA(cudaMalloc((void **)&m->nbr_sorted, sizeof(int32_t) * np), "identity map");
  T2SC_CUDA(cudaMalloc((void **)&m->tile_mask, sizeof(uint32_t) * (size_t)(m->ntiles > 0 ? m->ntiles : 1)),
            "identity map");
  if (n > 0) {
    identity_map_kernel<<<nblk(m->n_pad, 256), 256, 0, ctx->stream>>>(n, m->n_pad, m->nbr, m->mask, m->perm,
                                                                      m->nbr_sorted, m->tile_mask);
    T2SC_LAUNCHED(ctx, "identity_map");
  }
  *out = m.release();
  return T2SC_OK;
}

int build_map(t2sc_coords *c, int kd, int kh, int kw, int dil, t2sc_map **out, std::string &err) {
  auto key = std::make_tuple(kd, kh, kw, dil);
  auto it = c->maps.find(key);
  if (it != c->maps.end()) {
    *out = it->second;
    return T2SC_OK;
  }
  t2sc_ctx *ctx = c->ctx;
  cudaStream_t st = ctx->stream;
  std::unique_ptr<t2sc_map, void (*)(t2sc_map *)> m(new t2sc_map(), free_map);
  const int64_t n = c->n_targets;
  m->kvol = kd * kh * kw;
  m->n = n;
  m->n_src = c->n;
  m->ntiles = (n + kTileRows - 1) / kTileRows;
  m->n_pad = m->ntiles * kTileRows;
  const int K = m->kvol;
  T2SC_CUDA(cudaMalloc((void **)&m->nbr, sizeof(int32_t) * (size_t)K * (size_t)(n > 0 ? n : 1)), "map nbr");
  T2SC_CUDA(cudaMalloc((void **)&m->mask, sizeof(uint32_t) * (size_t)(n > 0 ? n : 1)), "map mask");
  T2SC_CUDA(cudaMalloc((void **)&m->perm, sizeof(int32_t) * (size_t)(m->n_pad > 0 ? m->n_pad : 1)), "map perm");
  T2SC_CUDA(cudaMalloc((void **)&m->nbr_sorted, sizeof(int32_t) * (size_t)K * (size_t)(m->n_pad > 0 ? m->n_pad : 1)),
            "map nbr_sorted");
  T2SC_CUDA(cudaMalloc((void **)&m->tile_mask, sizeof(uint32_t) * (size_t)(m->ntiles > 0 ? m->ntiles : 1)),
            "map tile_mask");
  if (n > 0) {
    unsigned long long *d_e = nullptr;
    uint32_t *mask_sorted = nullptr;
    int32_t *iota = nullptr, *perm_tmp = nullptr;
    void *temp = nullptr;
    size_t temp_bytes = 0;
    T2SC_CUDA(cudaMallocAsync((void **)&d_e, sizeof(unsigned long long), st), "map scratch");
    T2SC_CUDA(cudaMemsetAsync(d_e, 0, sizeof(unsigned long long), st), "map scratch");
    neighbor_map_kernel<<<nblk(n, 128), 128, 0, st>>>((const int4 *)c->d_coords + c->target_begin, n, c->d_keys, c->d_vals,
                                                       c->hcap - 1, kd, kh, kw, dil, m->nbr, m->mask, d_e);
    T2SC_LAUNCHED(ctx, "neighbor_map");
    T2SC_CUDA(cudaMallocAsync((void **)&mask_sorted, sizeof(uint32_t) * n, st), "sort scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&iota, sizeof(int32_t) * n, st), "sort scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&perm_tmp, sizeof(int32_t) * n, st), "sort scratch");
    iota_kernel<<<nblk(n, 256), 256, 0, st>>>(iota, n);
    T2SC_LAUNCHED(ctx, "iota");
    // stable LSD radix sort of rows by their occupancy mask
    T2SC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, m->mask, mask_sorted, iota, perm_tmp, (int)n, 0,
                                              K, st),
              "sort size");
    T2SC_CUDA(cudaMallocAsync(&temp, temp_bytes, st), "sort scratch");
    T2SC_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, m->mask, mask_sorted, iota, perm_tmp, (int)n, 0, K,
                                              st),
              "sort");
    ctx->launches += 2 * ((K + 7) / 8) + 2;  // approximate CUB launch count (onesweep passes)
    sorted_tiles_kernel<<<(unsigned)m->ntiles, kTileRows, 0, st>>>(m->nbr, m->mask, perm_tmp, n, m->n_pad, K,
                                                                    m->perm, m->nbr_sorted, m->tile_mask);
    T2SC_LAUNCHED(ctx, "sorted_tiles");
    unsigned long long e = 0;
    T2SC_CUDA(cudaMemcpyAsync(&e, d_e, sizeof(e), cudaMemcpyDeviceToHost, st), "map edge count");
    cudaFreeAsync(temp, st);
    cudaFreeAsync(perm_tmp, st);
    cudaFreeAsync(iota, st);
    cudaFreeAsync(mask_sorted, st);
    cudaFreeAsync(d_e, st);
    T2SC_CUDA(cudaStreamSynchronize(st), "map build");
    m->n_edges = (int64_t)e;
  }
  *out = m.get();
  c->maps[key] = m.release();
  return T2SC_OK;
}

int export_edges(t2sc_coords *c, t2sc_map *m, int64_t *src, int64_t *tgt, int64_t *kidx, std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  cudaStream_t st = ctx->stream;
  const int64_t total = (int64_t)m->kvol * m->n, E = m->n_edges;
  if (E == 0) return T2SC_OK;
  int32_t *flags = nullptr;
  int64_t *pos = nullptr, *d_out = nullptr;
  T2SC_CUDA(cudaMallocAsync((void **)&flags, sizeof(int32_t) * total, st), "export scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&pos, sizeof(int64_t) * total, st), "export scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_out, sizeof(int64_t) * 3 * E, st), "export scratch");
  edge_flags_kernel<<<nblk(total, 256), 256, 0, st>>>(m->nbr, total, flags);
  T2SC_LAUNCHED(ctx, "edge_flags");
  int rc = scan_counts(ctx, flags, total, pos, nullptr);
  if (rc != T2SC_OK) return rc;
  edge_emit_kernel<<<nblk(total, 256), 256, 0, st>>>(m->nbr, m->n, total, pos, d_out, d_out + E, d_out + 2 * E);
  T2SC_LAUNCHED(ctx, "edge_emit");
  T2SC_CUDA(cudaMemcpyAsync(src, d_out, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  T2SC_CUDA(cudaMemcpyAsync(tgt, d_out + E, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  T2SC_CUDA(cudaMemcpyAsync(kidx, d_out + 2 * E, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  cudaFreeAsync(flags, st);
  cudaFreeAsync(pos, st);
  cudaFreeAsync(d_out, st);
  T2SC_CUDA(cudaStreamSynchronize(st), "export");
  return T2SC_OK;
}

int export_csr(t2sc_coords *c, t2sc_map *m, int64_t *row_start, int64_t *src_s, int64_t *kidx_s,
               std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  cudaStream_t st = ctx->stream;
  const int64_t n = m->n, E = m->n_edges;
  int32_t *cnt = nullptr;
  int64_t *d_rs = nullptr, *d_out = nullptr;
  T2SC_CUDA(cudaMallocAsync((void **)&cnt, sizeof(int32_t) * (n + 1), st), "csr scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_rs, sizeof(int64_t) * (n + 1), st), "csr scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_out, sizeof(int64_t) * (2 * E + 1), st), "csr scratch");
  if (n > 0) {
    row_counts_kernel<<<nblk(n, 256), 256, 0, st>>>(m->mask, n, cnt);
    T2SC_LAUNCHED(ctx, "row_counts");
  }
  int rc = scan_counts(ctx, cnt, n, d_rs, d_rs + n);
  if (rc != T2SC_OK) return rc;
  if (n > 0) {
    csr_emit_kernel<<<nblk(n, 256), 256, 0, st>>>(m->nbr, m->mask, n, d_rs, d_out, d_out + E);
    T2SC_LAUNCHED(ctx, "csr_emit");
  }
  T2SC_CUDA(cudaMemcpyAsync(row_start, d_rs, sizeof(int64_t) * (n + 1), cudaMemcpyDeviceToHost, st), "csr copy");
  if (E > 0) {
    T2SC_CUDA(cudaMemcpyAsync(src_s, d_out, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "csr copy");
    T2SC_CUDA(cudaMemcpyAsync(kidx_s, d_out + E, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "csr copy");
  }
  cudaFreeAsync(cnt, st);
  cudaFreeAsync(d_rs, st);
  cudaFreeAsync(d_out, st);
  T2SC_CUDA(cudaStreamSynchronize(st), "csr export");
  return T2SC_OK;
}

}  // namespace t2sc
