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
// factor <= 0.25; nbr[k][r] (k-major, -1 = miss) so that one offset of a
// 128-row tile is one contiguous 512-byte read; a 32-bit occupancy mask per
// row. For the conv, rows are stably radix-sorted by that mask with its
// bits reordered (offsets farthest from the kernel centre most significant),
// so that rows with the same neighbour pattern share a tile and a tile only
// visits the offsets some of its rows use.
#include <cub/device/device_radix_sort.cuh>

#include "internal.h"

namespace t2sc {
namespace {

constexpr int64_t kEmpty = -1;
// Table capacity: the power of two >= 4 slots per row (load factor 1/8 to
// 1/4). Against 2 slots per row this shortens the linear-probe runs, misses
// above all: cfg4 map build 0.40 -> 0.32 ms, cfg5 0.92 vs 1.09 ms, the
// trilinear sampler 0.33 -> 0.25 ms, for 64 bytes of table per row.
constexpr uint64_t kHashSlotsPerRow = 4;

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

// Home slot of a key. (Grouping the 8 keys of a z / 8 column segment into
// one 128-byte line was measured slower: 0.57 vs 0.41 ms for the cfg4 map,
// longer probe runs and contended insert atomics.)
__device__ __forceinline__ uint64_t home_slot(uint64_t key, uint64_t hmask) { return mix64(key) & hmask; }

__global__ void hash_insert_kernel(const int4 *__restrict__ coords, int64_t n, longlong2 *slots, uint64_t hmask,
                                   int *err) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  int4 c = coords[r];
  if (c.x < 0 || c.y < -512 || c.y >= 1536 || c.z < -512 || c.z >= 1536 || c.w < -512 || c.w >= 1536) {
    atomicOr(err, kDevErrRange);
    return;
  }
  unsigned long long key = (unsigned long long)pack_key(c.x, c.y, c.z, c.w);
  uint64_t s = home_slot(key, hmask);
  for (uint64_t probe = 0; probe <= hmask; probe++) {
    unsigned long long *kp = reinterpret_cast<unsigned long long *>(&slots[s].x);
    unsigned long long prev = atomicCAS(kp, (unsigned long long)kEmpty, key);
    if (prev == (unsigned long long)kEmpty || prev == key) {
      atomicMax(reinterpret_cast<int *>(&slots[s].y), (int32_t)r);  // the last row with this key wins
      return;
    }
    s = (s + 1) & hmask;
  }
  atomicOr(err, kDevErrHashFull);
}

__device__ __forceinline__ int32_t hash_find(const longlong2 *__restrict__ slots, uint64_t hmask, int64_t key) {
  if (key == kEmpty) return -1;
  uint64_t s = home_slot((uint64_t)key, hmask);
  for (uint64_t probe = 0; probe <= hmask; probe++) {
    const longlong2 e = slots[s];  // key and row in one 16-byte load
    if (e.x == key) return (int32_t)e.y;
    if (e.x == kEmpty) return -1;
    s = (s + 1) & hmask;
  }
  return -1;
}

// Offset k of a kd x kh x kw kernel moves columns 1, 2, 3 by these amounts.
__device__ __forceinline__ void offset_of(int k, int kd, int kh, int kw, int dil, int64_t &o1, int64_t &o2,
                                          int64_t &o3) {
  const int kz = k / (kh * kw), ky = (k / kw) % kh, kx = k % kw;
  o1 = (int64_t)(kz - kd / 2) * dil;
  o2 = (int64_t)(ky - kh / 2) * dil;
  o3 = (int64_t)(kx - kw / 2) * dil;
}

// Pass 1: neighbours and occupancy mask of every target row. One warp per
// row, lane k probes offset k, so the 27 probes of a row are in flight
// together; the row's results are one 128-byte line of rows32 [n][32]; the
// warp's ballot is the row's mask. Edges are counted per block, then added
// once to *n_edges.
__global__ void __launch_bounds__(256) row_mask_kernel(const int4 *__restrict__ coords, int64_t n,
                                                       const longlong2 *__restrict__ slots, uint64_t hmask, int kd,
                                                       int kh, int kw, int dil, uint32_t *__restrict__ mask,
                                                       uint32_t *__restrict__ sort_key, int32_t *__restrict__ rows32,
                                                       unsigned long long *__restrict__ n_edges) {
  __shared__ unsigned block_edges;
  if (threadIdx.x == 0) block_edges = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, K = kd * kh * kw;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  unsigned cnt = 0;
  int64_t o1 = 0, o2 = 0, o3 = 0;
  if (lane < K) offset_of(lane, kd, kh, kw, dil, o1, o2, o3);
  // Sort-key bit of this lane's offset: offsets ordered by distance from the
  // kernel centre, farthest (rarest in a sparse set) in the most significant
  // bits. Rows with the same mask still sort together; among different
  // masks, rows that differ only in rare offsets land in the same tile, which
  // shrinks tile unions on sparse sets (cfg5: 6.7 % fewer tile x offset pairs).
  const int dist = lane < K ? abs(lane / (kh * kw) - kd / 2) + abs((lane / kw) % kh - kh / 2) + abs(lane % kw - kw / 2)
                            : -1;
  int before = 0;
  for (int j = 0; j < K; j++) {
    const int dj = __shfl_sync(0xffffffffu, dist, j);
    before += (dj > dist || (dj == dist && j < lane)) ? 1 : 0;
  }
  const uint32_t key_bit = lane < K ? 1u << (K - 1 - before) : 0u;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
    const int4 c = coords[r];
    const int32_t src = lane < K ? hash_find(slots, hmask, pack_key(c.x, c.y + o1, c.z + o2, c.w + o3)) : -1;
    rows32[r * 32 + lane] = src;  // one 128-byte line per row
    const uint32_t m = __ballot_sync(0xffffffffu, src >= 0);
    const uint32_t key = __reduce_or_sync(0xffffffffu, src >= 0 ? key_bit : 0u);
    if (lane == 0) {
      mask[r] = m;
      sort_key[r] = key;
      cnt += __popc(m);
    }
  }
  if (lane == 0 && cnt) atomicAdd(&block_edges, cnt);
  __syncthreads();
  if (threadIdx.x == 0 && block_edges) atomicAdd(n_edges, (unsigned long long)block_edges);
}

// Pass 2 (after rows are sorted by their mask keys): neighbour rows in sorted order.
// One 128-thread block per tile: each warp reads the 128-byte result lines
// of 32 of the tile's rows (one coalesced line per row), the block
// transposes them in shared memory and writes nbr_sorted[k][tile rows] as
// one 512-byte run per offset; it also writes the padded permutation and
// the tile's offset mask.
__global__ void __launch_bounds__(kTileRows) sorted_nbr_kernel(int64_t n, int64_t n_pad, int kvol,
                                                              const int32_t *__restrict__ sorted_rows,
                                                              const uint32_t *__restrict__ mask,
                                                              const int32_t *__restrict__ rows32,
                                                              int32_t *__restrict__ perm_out,
                                                              int32_t *__restrict__ nbr_sorted,
                                                              uint32_t *__restrict__ tile_mask) {
  __shared__ int32_t tr[32][kTileRows + 1];
  __shared__ uint32_t wm[kTileRows / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t base = (int64_t)blockIdx.x * kTileRows;
  for (int i = 0; i < 32; i++) {
    const int pl = warp * 32 + i;
    const int64_t p = base + pl;
    const int32_t row = p < n ? sorted_rows[p] : -1;
    tr[lane][pl] = row >= 0 ? rows32[(int64_t)row * 32 + lane] : -1;
  }
  const int64_t p = base + threadIdx.x;
  const int32_t row = p < n ? sorted_rows[p] : -1;
  perm_out[p] = row;
  const uint32_t m = __reduce_or_sync(0xffffffffu, row >= 0 ? mask[row] : 0u);
  if (lane == 0) wm[warp] = m;
  __syncthreads();
  for (int k = 0; k < kvol; k++) nbr_sorted[(int64_t)k * n_pad + p] = tr[k][threadIdx.x];
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int i = 0; i < kTileRows / 32; i++) t |= wm[i];
    tile_mask[blockIdx.x] = t;
  }
}

// pos[perm[p]] = p: sorted position of every target row (for the exports,
// which list edges in the reference's row order).
__global__ void inverse_perm_kernel(const int32_t *__restrict__ perm, int64_t n_pad, int32_t *__restrict__ pos) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p < n_pad) {
    const int32_t r = perm[p];
    if (r >= 0) pos[r] = (int32_t)p;
  }
}

__global__ void iota_kernel(int32_t *v, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = (int32_t)i;
}


__global__ void edge_flags_kernel(const int32_t *__restrict__ nbr_sorted, const int32_t *__restrict__ pos, int64_t n,
                                  int64_t n_pad, int64_t total, int32_t *__restrict__ flags) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) flags[i] = nbr_sorted[(i / n) * n_pad + pos[i % n]] >= 0 ? 1 : 0;
}

// Edges in the reference order: offset-major, target ascending (i = k*n + r).
__global__ void edge_emit_kernel(const int32_t *__restrict__ nbr_sorted, const int32_t *__restrict__ pos, int64_t n,
                                 int64_t n_pad, int64_t total, const int64_t *__restrict__ out_pos,
                                 int64_t *__restrict__ src, int64_t *__restrict__ tgt, int64_t *__restrict__ kidx) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int64_t k = i / n, r = i % n;
  int32_t s = nbr_sorted[k * n_pad + pos[r]];
  if (s < 0) return;
  int64_t p = out_pos[i];
  src[p] = s;
  tgt[p] = r;
  kidx[p] = k;
}

__global__ void row_counts_kernel(const uint32_t *__restrict__ mask, int64_t n, int32_t *__restrict__ cnt) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) cnt[r] = __popc(mask[r]);
}

// CSR rows in target order, kernel index ascending within a row.
__global__ void csr_emit_kernel(const int32_t *__restrict__ nbr_sorted, const int32_t *__restrict__ pos,
                                const uint32_t *__restrict__ mask, int64_t n, int64_t n_pad,
                                const int64_t *__restrict__ row_start, int64_t *__restrict__ src_s,
                                int64_t *__restrict__ kidx_s) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  uint32_t m = mask[r];
  const int64_t q = pos[r];
  int64_t p = row_start[r];
  while (m) {
    int k = __ffs(m) - 1;
    m &= m - 1;
    src_s[p] = nbr_sorted[(int64_t)k * n_pad + q];
    kidx_s[p] = k;
    p++;
  }
}

inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

// Trilinear sample of sparse voxel features at query points given in voxel
// units (trellis2_mojo/meshing/vertex_attrs.mojo:46-104, the flex_gemm
// grid_sample_3d semantics): the 8 neighbours are p +- 0.5 truncated toward
// zero (for p < 0.5 two of them truncate to the same voxel and both count),
// each weighs prod(1 - |n + 0.5 - p|); voxels absent from the set, negative
// or >= grid_size weigh 0; the result is renormalised by the weight sum
// clamped to 1e-12. Arithmetic in f32 in the reference's order (neighbours
// k = 0..7 with x the slowest offset, the channel sums in k order), with the
// roundings written out so that no multiply-add is contracted.
// Eight lanes per query: lane k probes neighbour k, so the eight hash
// probes of a query are in flight together; the weight sum and the channel
// sums are then formed in neighbour order from shuffled (row, weight) pairs,
// lane k producing channels k, k + 8, ... A missing neighbour adds an exact
// 0 to the weight sum, which leaves it unchanged.
__global__ void __launch_bounds__(256) grid_sample_kernel(const longlong2 *__restrict__ slots, uint64_t hmask,
                                                          const float *__restrict__ feats, int c, int grid_size,
                                                          const float *__restrict__ query, int64_t l,
                                                          float *__restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t q = t >> 3;
  const int k = threadIdx.x & 7, lead = (threadIdx.x & 31) & ~7;
  int32_t idx = -1;
  float w = 0.f;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (q < l) {
    px = query[3 * q], py = query[3 * q + 1], pz = query[3 * q + 2];
    const float ox = (k & 4) ? 0.5f : -0.5f, oy = (k & 2) ? 0.5f : -0.5f, oz = (k & 1) ? 0.5f : -0.5f;
    const float fx = __fadd_rn(px, ox), fy = __fadd_rn(py, oy), fz = __fadd_rn(pz, oz);
    // a value that truncates below 0 or reaches grid_size names no voxel
    if (fx > -1.f && fy > -1.f && fz > -1.f && fx < (float)grid_size && fy < (float)grid_size &&
        fz < (float)grid_size) {
      const int nx = (int)fx, ny = (int)fy, nz = (int)fz;  // truncation toward zero
      const int32_t r = hash_find(slots, hmask, pack_key(0, nx, ny, nz));
      if (r >= 0) {
        const float wx = __fsub_rn(1.f, fabsf(__fsub_rn(__fadd_rn((float)nx, 0.5f), px)));
        const float wy = __fsub_rn(1.f, fabsf(__fsub_rn(__fadd_rn((float)ny, 0.5f), py)));
        const float wz = __fsub_rn(1.f, fabsf(__fsub_rn(__fadd_rn((float)nz, 0.5f), pz)));
        idx = r;
        w = __fmul_rn(__fmul_rn(wx, wy), wz);
      }
    }
  }
  float wsum = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, w, lead + j));
  const float denom = wsum < 1e-12f ? 1e-12f : wsum;
  for (int c0 = 0; c0 < c; c0 += 8) {
    const int ch = c0 + k;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int32_t rj = __shfl_sync(0xffffffffu, idx, lead + j);
      const float wj = __shfl_sync(0xffffffffu, w, lead + j);
      if (rj >= 0 && ch < c) acc = __fadd_rn(acc, __fmul_rn(wj, feats[(int64_t)rj * c + ch]));
    }
    if (q < l && ch < c) out[q * c + ch] = __fdiv_rn(acc, denom);
  }
}

}  // namespace

int build_hash(t2sc_coords *c, std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  uint64_t cap = 1024;
  while (cap < kHashSlotsPerRow * (uint64_t)c->n) cap <<= 1;
  c->hcap = cap;
  T2SC_CUDA(cudaMallocAsync((void **)&c->d_slots, cap * sizeof(longlong2), ctx->stream), "hash slots");
  // every byte 0xff: keys and rows read as -1 (empty)
  T2SC_CUDA(cudaMemsetAsync(c->d_slots, 0xff, cap * sizeof(longlong2), ctx->stream), "hash init");
  if (c->n > 0) {
    hash_insert_kernel<<<nblk(c->n, 256), 256, 0, ctx->stream>>>((const int4 *)c->d_coords, c->n, c->d_slots,
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
  cudaStream_t st = m->ctx ? m->ctx->stream : nullptr;
  cudaFreeAsync(m->d_edges, st);
  cudaFreeAsync(m->mask, st);
  cudaFreeAsync(m->perm, st);
  cudaFreeAsync(m->nbr_sorted, st);
  cudaFreeAsync(m->tile_mask, st);
  delete m;
}

int map_edges(t2sc_map *m, int64_t *n_edges, std::string &err) {
  if (m->n_edges < 0) {
    unsigned long long e = 0;
    if (m->d_edges) {
      T2SC_CUDA(cudaMemcpyAsync(&e, m->d_edges, sizeof(e), cudaMemcpyDeviceToHost, m->ctx->stream), "edge count");
      T2SC_CUDA(cudaStreamSynchronize(m->ctx->stream), "edge count");
    }
    m->n_edges = (int64_t)e;
  }
  *n_edges = m->n_edges;
  return T2SC_OK;
}

// Allocates the arrays of a map with n target rows and kvol offsets from
// the stream-ordered pool.
static int alloc_map(t2sc_ctx *ctx, t2sc_map *m, int64_t n, int kvol, std::string &err) {
  cudaStream_t st = ctx->stream;
  m->ctx = ctx;
  m->kvol = kvol;
  m->n = n;
  m->ntiles = (n + kTileRows - 1) / kTileRows;
  m->n_pad = m->ntiles * kTileRows;
  const size_t np = (size_t)(m->n_pad > 0 ? m->n_pad : 1), nn = (size_t)(n > 0 ? n : 1);
  T2SC_CUDA(cudaMallocAsync((void **)&m->d_edges, sizeof(unsigned long long), st), "map");
  T2SC_CUDA(cudaMallocAsync((void **)&m->mask, sizeof(uint32_t) * nn, st), "map mask");
  T2SC_CUDA(cudaMallocAsync((void **)&m->perm, sizeof(int32_t) * np, st), "map perm");
  T2SC_CUDA(cudaMallocAsync((void **)&m->nbr_sorted, sizeof(int32_t) * (size_t)kvol * np, st), "map nbr_sorted");
  T2SC_CUDA(cudaMallocAsync((void **)&m->tile_mask, sizeof(uint32_t) * (size_t)(m->ntiles > 0 ? m->ntiles : 1), st),
            "map tile_mask");
  T2SC_CUDA(cudaMemsetAsync(m->d_edges, 0, sizeof(unsigned long long), st), "map");
  return T2SC_OK;
}

__global__ void identity_map_kernel(int64_t n, int64_t n_pad, uint32_t *__restrict__ mask, int32_t *__restrict__ perm,
                                    int32_t *__restrict__ nbr_sorted, uint32_t *__restrict__ tile_mask) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_pad) return;
  const int32_t r = p < n ? (int32_t)p : -1;
  perm[p] = r;
  nbr_sorted[p] = r;
  if (p < n) mask[p] = 1u;
  if (p % kTileRows == 0) tile_mask[p / kTileRows] = 1u;  // every tile holds >= 1 row
}

int build_identity_map(t2sc_ctx *ctx, int64_t n, t2sc_map **out, std::string &err) {
  std::unique_ptr<t2sc_map, void (*)(t2sc_map *)> m(new t2sc_map(), free_map);
  int rc = alloc_map(ctx, m.get(), n, 1, err);
  if (rc != T2SC_OK) return rc;
  m->n_src = m->n_edges = n;
  if (n > 0) {
    identity_map_kernel<<<nblk(m->n_pad, 256), 256, 0, ctx->stream>>>(n, m->n_pad, m->mask, m->perm, m->nbr_sorted,
                                                                      m->tile_mask);
    T2SC_LAUNCHED(ctx, "identity_map");
  }
  *out = m.release();
  return T2SC_OK;
}

// Neighbour map of a coordinate set, entirely stream-ordered (no host
// synchronisation): neighbours and masks per row (one warp per row), rows
// sorted by mask key into 128-row tiles, then the neighbour rows transposed
// into the sorted [K][n_pad] layout.
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
  const int K = kd * kh * kw;
  int rc = alloc_map(ctx, m.get(), n, K, err);
  if (rc != T2SC_OK) return rc;
  m->n_src = c->n;
  if (n == 0) m->n_edges = 0;
  if (n > 0) {
    const int4 *tc = (const int4 *)c->d_coords + c->target_begin;
    const int warps_per_block = 8;
    const int64_t blocks = std::min<int64_t>((n + warps_per_block - 1) / warps_per_block, (int64_t)ctx->num_sms * 64);
    int32_t *rows32 = nullptr;
    uint32_t *sort_key = nullptr;
    T2SC_CUDA(cudaMallocAsync((void **)&rows32, sizeof(int32_t) * 32 * n, st), "map scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&sort_key, sizeof(uint32_t) * n, st), "map scratch");
    row_mask_kernel<<<(unsigned)blocks, 32 * warps_per_block, 0, st>>>(tc, n, c->d_slots, c->hcap - 1, kd, kh, kw,
                                                                       dil, m->mask, sort_key, rows32, m->d_edges);
    T2SC_LAUNCHED(ctx, "row_mask");
    int32_t *iota = nullptr, *sorted = nullptr;
    void *temp = nullptr;
    size_t temp_bytes = 0;
    T2SC_CUDA(cudaMallocAsync((void **)&iota, sizeof(int32_t) * n, st), "sort scratch");
    T2SC_CUDA(cudaMallocAsync((void **)&sorted, sizeof(int32_t) * n, st), "sort scratch");
    iota_kernel<<<nblk(n, 256), 256, 0, st>>>(iota, n);
    T2SC_LAUNCHED(ctx, "iota");
    // stable LSD radix sort of rows by their occupancy mask (K key bits):
    // rows with the same neighbour pattern share tiles, so a tile visits few
    // offsets (89 % of the issued MMA rows useful at the 512^3 shell, 42 %
    // in coordinate order)
    uint32_t *mask_sorted = nullptr;
    T2SC_CUDA(cudaMallocAsync((void **)&mask_sorted, sizeof(uint32_t) * n, st), "sort scratch");
    T2SC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, sort_key, mask_sorted, iota, sorted, (int)n, 0, K,
                                              st),
              "sort size");
    T2SC_CUDA(cudaMallocAsync(&temp, temp_bytes, st), "sort scratch");
    T2SC_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, sort_key, mask_sorted, iota, sorted, (int)n, 0, K, st),
              "sort");
    ctx->launches += 2 * ((K + 7) / 8) + 2;  // approximate CUB launch count (onesweep passes)
    cudaFreeAsync(mask_sorted, st);
    cudaFreeAsync(sort_key, st);
    sorted_nbr_kernel<<<(unsigned)m->ntiles, kTileRows, 0, st>>>(n, m->n_pad, K, sorted, m->mask, rows32, m->perm,
                                                                 m->nbr_sorted, m->tile_mask);
    T2SC_LAUNCHED(ctx, "sorted_nbr");
    cudaFreeAsync(rows32, st);
    if (temp) cudaFreeAsync(temp, st);
    cudaFreeAsync(sorted, st);
    cudaFreeAsync(iota, st);
  }
  *out = m.get();
  c->maps[key] = m.release();
  return T2SC_OK;
}

// Sorted position of every target row (stream-ordered scratch).
static int map_positions(t2sc_ctx *ctx, t2sc_map *m, int32_t **pos, std::string &err) {
  T2SC_CUDA(cudaMallocAsync((void **)pos, sizeof(int32_t) * (size_t)(m->n > 0 ? m->n : 1), ctx->stream),
            "export scratch");
  if (m->n_pad > 0) {
    inverse_perm_kernel<<<nblk(m->n_pad, 256), 256, 0, ctx->stream>>>(m->perm, m->n_pad, *pos);
    T2SC_LAUNCHED(ctx, "inverse_perm");
  }
  return T2SC_OK;
}

int export_edges(t2sc_coords *c, t2sc_map *m, int64_t *src, int64_t *tgt, int64_t *kidx, std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  cudaStream_t st = ctx->stream;
  const int64_t total = (int64_t)m->kvol * m->n;
  int64_t E = 0;
  int rc = map_edges(m, &E, err);
  if (rc != T2SC_OK) return rc;
  if (E == 0) return T2SC_OK;
  int32_t *flags = nullptr, *pos = nullptr;
  int64_t *opos = nullptr, *d_out = nullptr;
  if ((rc = map_positions(ctx, m, &pos, err)) != T2SC_OK) return rc;
  T2SC_CUDA(cudaMallocAsync((void **)&flags, sizeof(int32_t) * total, st), "export scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&opos, sizeof(int64_t) * total, st), "export scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_out, sizeof(int64_t) * 3 * E, st), "export scratch");
  edge_flags_kernel<<<nblk(total, 256), 256, 0, st>>>(m->nbr_sorted, pos, m->n, m->n_pad, total, flags);
  T2SC_LAUNCHED(ctx, "edge_flags");
  rc = scan_counts(ctx, flags, total, opos, nullptr);
  if (rc != T2SC_OK) return rc;
  edge_emit_kernel<<<nblk(total, 256), 256, 0, st>>>(m->nbr_sorted, pos, m->n, m->n_pad, total, opos, d_out,
                                                     d_out + E, d_out + 2 * E);
  T2SC_LAUNCHED(ctx, "edge_emit");
  T2SC_CUDA(cudaMemcpyAsync(src, d_out, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  T2SC_CUDA(cudaMemcpyAsync(tgt, d_out + E, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  T2SC_CUDA(cudaMemcpyAsync(kidx, d_out + 2 * E, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, st), "export copy");
  cudaFreeAsync(flags, st);
  cudaFreeAsync(opos, st);
  cudaFreeAsync(d_out, st);
  cudaFreeAsync(pos, st);
  T2SC_CUDA(cudaStreamSynchronize(st), "export");
  return T2SC_OK;
}

int export_csr(t2sc_coords *c, t2sc_map *m, int64_t *row_start, int64_t *src_s, int64_t *kidx_s,
               std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  cudaStream_t st = ctx->stream;
  const int64_t n = m->n;
  int64_t E = 0;
  int rc = map_edges(m, &E, err);
  if (rc != T2SC_OK) return rc;
  int32_t *cnt = nullptr, *pos = nullptr;
  int64_t *d_rs = nullptr, *d_out = nullptr;
  if ((rc = map_positions(ctx, m, &pos, err)) != T2SC_OK) return rc;
  T2SC_CUDA(cudaMallocAsync((void **)&cnt, sizeof(int32_t) * (n + 1), st), "csr scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_rs, sizeof(int64_t) * (n + 1), st), "csr scratch");
  T2SC_CUDA(cudaMallocAsync((void **)&d_out, sizeof(int64_t) * (2 * E + 1), st), "csr scratch");
  if (n > 0) {
    row_counts_kernel<<<nblk(n, 256), 256, 0, st>>>(m->mask, n, cnt);
    T2SC_LAUNCHED(ctx, "row_counts");
  }
  rc = scan_counts(ctx, cnt, n, d_rs, d_rs + n);
  if (rc != T2SC_OK) return rc;
  if (n > 0) {
    csr_emit_kernel<<<nblk(n, 256), 256, 0, st>>>(m->nbr_sorted, pos, m->mask, n, m->n_pad, d_rs, d_out, d_out + E);
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
  cudaFreeAsync(pos, st);
  T2SC_CUDA(cudaStreamSynchronize(st), "csr export");
  return T2SC_OK;
}

int grid_sample_device(t2sc_coords *c, const float *feats, int ch, int grid_size, const float *query, int64_t l,
                       float *out, std::string &err) {
  t2sc_ctx *ctx = c->ctx;
  if (l == 0) return T2SC_OK;
  grid_sample_kernel<<<nblk(l * 8, 256), 256, 0, ctx->stream>>>(c->d_slots, c->hcap - 1, feats, ch, grid_size, query, l,
                                                          out);
  T2SC_LAUNCHED(ctx, "grid_sample");
  return T2SC_OK;
}

}  // namespace t2sc
