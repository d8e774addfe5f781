// Internal declarations shared by the libt2sc translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/t2sc.h"

namespace t2sc {

constexpr int kTileRows = 128;  // output rows per conv tile (UMMA M)
constexpr int kMaxK = 32;       // kernel volume must fit a 32-bit offset mask

// Device-side error flags (bit set by kernels, read by the host after a
// launch sequence). Kernels never trap; they record and return.
enum DevErr : int {
  kDevErrRange = 1,       // coordinate outside [-512, 1536) or batch < 0
  kDevErrHashFull = 2,    // probe sequence exhausted (cannot happen at load <= 0.5)
  kDevErrTimeout = 4,     // bounded mbarrier wait gave up
  kDevErrInternal = 8,
};

struct Status {
  int code = T2SC_OK;
  std::string msg;
};

}  // namespace t2sc

struct t2sc_map;

struct t2sc_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  int *d_err = nullptr;      // device error flags (one int)
  int64_t launches = 0;      // kernels launched by this context
  std::string last_error;
  // identity row maps of the linear layers, one per row count, shared by
  // every linear handle of the context and kept until it is destroyed
  std::map<int64_t, t2sc_map *> id_maps;
  // grow-only scratch buffers ([0]: the split-TF32 hi/lo parts of a conv input)
  void *stage[4] = {nullptr, nullptr, nullptr, nullptr};
  size_t stage_cap[4] = {0, 0, 0, 0};
  // copy streams of the pipelined conv chain (created on first use)
  cudaStream_t up_stream = nullptr, down_stream = nullptr;
};

// One neighbour map for a (kernel, dilation) on a coordinate set. Device
// arrays come from the context's stream-ordered pool (no synchronising
// allocation) and are released on the context's stream.
struct t2sc_map {
  t2sc_ctx *ctx = nullptr;
  int kvol = 27;
  int64_t n = 0, n_pad = 0, ntiles = 0;  // n: target (output) rows
  int64_t n_src = 0;                      // rows of the input features (targets + halo)
  int64_t n_edges = -1;                   // edge count once read back (-1: still on the device)
  unsigned long long *d_edges = nullptr;  // device edge count
  uint32_t *mask = nullptr;      // [n]       bit k set iff target row r has a neighbour at offset k
  int32_t *perm = nullptr;       // [n_pad]   sorted position -> row (-1 padding)
  int32_t *nbr_sorted = nullptr; // [K][n_pad] source row of offset k for sorted position p (-1 = miss)
  uint32_t *tile_mask = nullptr; // [ntiles]  OR of masks in each 128-row tile
};

// One row slab of a pipelined conv chain (api.cu): local rows [lo, hi) of
// the parent coordinate set (own rows [t0, t1) plus a halo as deep as the
// chain's reach along x), a handle whose targets are all local rows and one
// whose targets are the own rows.
struct t2sc_chain_slab {
  int64_t lo = 0, t0 = 0, t1 = 0, hi = 0;
  t2sc_coords *all = nullptr, *own = nullptr;
};

struct t2sc_coords {
  t2sc_ctx *ctx = nullptr;
  int64_t n = 0;                 // all rows (targets first, then halo rows)
  int64_t n_targets = 0;         // rows that receive conv outputs
  int64_t target_begin = 0;      // first target row (targets are rows [target_begin, +n_targets))
  int32_t *d_coords = nullptr;   // [n,4]
  uint64_t hcap = 0;             // hash capacity (power of two)
  // [hcap] slots of 16 bytes: int64 key, int32 row, 4 bytes padding (a
  // probe reads key and row with one load)
  longlong2 *d_slots = nullptr;
  std::map<std::tuple<int, int, int, int>, t2sc_map *> maps;
  // pipelined-chain plans per x-reach (empty: this set is not pipelined)
  std::map<int64_t, std::vector<t2sc_chain_slab>> chain_plans;
};

struct t2sc_conv {
  t2sc_ctx *ctx = nullptr;
  int co = 0, ci = 0, kd = 3, kh = 3, kw = 3, kvol = 27, dilation = 1, dtype = 0;
  float *d_bias = nullptr;       // [co] (zeros when no bias)
  bool has_bias = false;
  // tensor-core operand image: pre-swizzled B blocks, one per
  // (co tile, k, ci chunk), each bn rows x row_bytes
  void *d_wtc = nullptr;
  int bn = 0, row_bytes = 0, nchunks = 0, nco_tiles = 0;
  int tc_path = 0;               // 1 = tcgen05 path, 0 = SIMT path
  float *d_w_simt = nullptr;     // [K][ci][co] f32 (SIMT path)
  void *d_w_lo = nullptr;        // split-TF32 low parts image (f32 mode)
};

namespace t2sc {
// ---- map building (hashmap.cu) ----
int build_hash(t2sc_coords *c, std::string &err);
int build_map(t2sc_coords *c, int kd, int kh, int kw, int dil, t2sc_map **out, std::string &err);
void free_map(t2sc_map *m);
// Edge count of a map (reads it back from the device once: synchronises).
int map_edges(t2sc_map *m, int64_t *n_edges, std::string &err);

// One-offset map with nbr[0][r] = r for rows [0, n): a linear layer run
// through the conv kernels (dense rows, no coordinates).
int build_identity_map(t2sc_ctx *ctx, int64_t n, t2sc_map **out, std::string &err);
int export_edges(t2sc_coords *c, t2sc_map *m, int64_t *src, int64_t *tgt, int64_t *kidx, std::string &err);
int export_csr(t2sc_coords *c, t2sc_map *m, int64_t *row_start, int64_t *src_s, int64_t *kidx_s,
               std::string &err);
// Trilinear sample of [n, ch] f32 features over the handle's hash (batch 0)
// at l query points (f32 [l, 3], voxel units) into out [l, ch].
int grid_sample_device(t2sc_coords *c, const float *feats, int ch, int grid_size, const float *query, int64_t l,
                       float *out, std::string &err);

// ---- exclusive scan of int32 counts into int64 offsets (scan.cu) ----
// out[i] = sum(in[0..i)), *total (device int64) = sum(in). Scratch is
// allocated stream-ordered on `stream` and released before return.
int scan_counts(t2sc_ctx *ctx, const int32_t *in, int64_t n, int64_t *out, int64_t *d_total);
// Same scan with caller-provided block-sum scratch of scan_block_count(n)
// int64 entries; allocates nothing.
constexpr int64_t kScanTileItems = 2048;  // items per scan block (256 threads x 8)
inline int64_t scan_block_count(int64_t n) { return (n + kScanTileItems - 1) / kScanTileItems; }
int scan_counts_into(t2sc_ctx *ctx, const int32_t *in, int64_t n, int64_t *out, int64_t *d_total,
                     int64_t *block_sums);

// ---- conv kernels ----
int conv_tc_prepare(t2sc_conv *cv, const float *w_host, std::string &err);
int conv_tc_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags,
                   const void *residual, std::string &err);
int conv_simt_prepare(t2sc_conv *cv, const float *w_host, std::string &err);

int conv_simt_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags,
                     const void *residual, std::string &err);

// ---- elementwise helpers (convert.cu) ----
int f32_to_dtype(t2sc_ctx *ctx, const float *in, void *out, int64_t count, int dtype);
int dtype_to_f32(t2sc_ctx *ctx, const void *in, float *out, int64_t count, int dtype);

// ---- subdivision (subdiv.cu) ----
int subdivide_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub, int keep_mode,
                     const void *feats, int c, int feats_mode, int dtype, int32_t *out_coords,
                     void *out_feats, int32_t *out_parent, int32_t *out_subidx, int64_t *m,
                     std::string &err);

// ---- LayerNorm (+ SiLU) (norm.cu) ----
int layernorm_device(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w, const float *b,
                     float eps, int flags, int dtype, std::string &err);

// ---- pipeline glue (pipeline.cu) ----
int fdg_head_device(t2sc_ctx *ctx, const float *feats, int64_t t, float margin, float *vertices, float *intersected,
                    float *quad, std::string &err);
int cascade_coords_device(t2sc_ctx *ctx, const int32_t *hr_coords, int64_t n, int lr_resolution, int resolution,
                          int64_t max_num_tokens, int32_t *out_coords, int64_t *num_tokens, int *hr_resolution,
                          std::string &err);

// ---- error-flag helpers (api.cu) ----
int read_dev_err(t2sc_ctx *ctx, int *flags);

inline int cuda_status(cudaError_t e, std::string &err, const char *what) {
  if (e == cudaSuccess) return T2SC_OK;
  err = std::string(what) + ": " + cudaGetErrorString(e);
  return e == cudaErrorMemoryAllocation ? T2SC_ERR_OOM : T2SC_ERR_CUDA;
}
}  // namespace t2sc

#define T2SC_CUDA(call, what)                                           \
  do {                                                                  \
    int _rc = t2sc::cuda_status((call), err, what);                     \
    if (_rc != T2SC_OK) return _rc;                                     \
  } while (0)

#define T2SC_LAUNCHED(ctx, what)                                        \
  do {                                                                  \
    (ctx)->launches++;                                                  \
    int _rc = t2sc::cuda_status(cudaGetLastError(), err, what);         \
    if (_rc != T2SC_OK) return _rc;                                     \
  } while (0)
