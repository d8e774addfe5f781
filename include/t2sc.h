/* t2sc — B200 (sm_100a) sparse submanifold convolution for TRELLIS.2-Mojo.
 *
 * C ABI of libt2sc.so. Every entry point returns an int status (T2SC_OK = 0)
 * and never aborts the process; t2sc_last_error() returns the message of the
 * last failure on a context. Plain pointers and sizes only.
 *
 * Reference interfaces replaced (paths inside the TRELLIS.2-Mojo project):
 *   SparseConv3d(weight [Co,Kd,Kh,Kw,Ci], bias, dilation)  trellis2_mojo/sparse/conv.mojo:31-47
 *   SparseConv3d._neighbor_map -> (src, tgt, kidx)          trellis2_mojo/sparse/conv.mojo:56-96
 *   CSR counting sort by target                             trellis2_mojo/sparse/conv.mojo:117-147
 *   SparseConv3d.forward                                    trellis2_mojo/sparse/conv.mojo:98-199
 *   GpuSparseConv.try_build / forward                       trellis2_mojo/gpu/conv.mojo:264-329, 334-477
 *   sparse_conv3d_from (attach point at model load)         trellis2_mojo/loaders.mojo:43-50
 *   SparseTensor coords int32 [N,4] (b,x,y,z) + spatial cache  trellis2_mojo/sparse/basic.mojo:296-339, 542-558
 *   SparseUpsample.forward_subdivision                      trellis2_mojo/sparse/spatial/basic.mojo:144-174
 *   SparseChannel2Spatial.forward_subdivision / _unfold     trellis2_mojo/sparse/spatial/spatial2channel.mojo:97-145
 *   _binarize (sub > 0)                                     trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:30-37
 *   activation(ACT_SILU): v / (1 + exp(-v))                 trellis2_mojo/modules/nn.mojo:567-568
 *
 * Threading: calls on one context are serialised by the caller (as the
 * reference's single GpuContext is); all device work of a context runs on
 * its stream. "_device" entry points take device pointers and are
 * asynchronous on that stream; the others take host pointers and return
 * after the results are in host memory.
 */
#ifndef T2SC_H
#define T2SC_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define T2SC_OK 0
#define T2SC_ERR_INVALID 1     /* bad argument or shape (reference: raise Error) */
#define T2SC_ERR_CUDA 2        /* a CUDA runtime call failed */
#define T2SC_ERR_OOM 3         /* device allocation failed */
#define T2SC_ERR_RANGE 4       /* coordinate outside the packable range [-512, 1536) or batch < 0 */
#define T2SC_ERR_TIMEOUT 5     /* a bounded device wait gave up; the context stays usable */
#define T2SC_ERR_UNSUPPORTED 6 /* shape not supported by this build */
#define T2SC_ERR_CAPACITY 7    /* caller's output buffer too small; required size returned */

/* ---- arithmetic modes (conv weights, inputs and outputs) ---- */
#define T2SC_DT_F32 0  /* f32 in/out, f32-accurate (split-TF32 tensor cores) */
#define T2SC_DT_F16 1  /* f16 in/out, f32 accumulate */
#define T2SC_DT_BF16 2 /* bf16 in/out, f32 accumulate */

/* ---- epilogue flags, applied in this order after the bias ---- */
#define T2SC_SILU 1     /* y = y / (1 + exp(-y)) */
#define T2SC_RESIDUAL 2 /* y += residual (same dtype and shape as y) */

/* ---- subdivision ---- */
#define T2SC_SUB_NONZERO 0  /* keep child c of row r iff sub[r*8+c] != 0 (forward_subdivision) */
#define T2SC_SUB_POSITIVE 1 /* keep iff sub[r*8+c] > 0 (_binarize then forward_subdivision) */
#define T2SC_FEATS_NONE 0     /* coordinates only */
#define T2SC_FEATS_UPSAMPLE 1 /* out[e] = x[parent]               (SparseUpsample) */
#define T2SC_FEATS_C2S 2      /* out[e] = x[parent, c*C:(c+1)*C]  (SparseChannel2Spatial) */

typedef struct t2sc_ctx t2sc_ctx;
typedef struct t2sc_coords t2sc_coords;
typedef struct t2sc_conv t2sc_conv;

/* ---- context: one per device (replaces GpuContext, gpu/context.mojo:116-165) ---- */
int t2sc_ctx_create(int device, t2sc_ctx **out);
int t2sc_ctx_destroy(t2sc_ctx *ctx);
/* Run this context's work on a caller-owned cudaStream_t (NULL restores the
 * context's own stream; cudaStreamLegacy, (void *)1, is the legacy default
 * stream). */
int t2sc_ctx_set_stream(t2sc_ctx *ctx, void *cuda_stream);
int t2sc_ctx_synchronize(t2sc_ctx *ctx);
const char *t2sc_last_error(const t2sc_ctx *ctx);
/* Kernel launches issued by this context since creation (diagnostics). */
int t2sc_ctx_launch_count(const t2sc_ctx *ctx, int64_t *count);
/* Device self-test (replaces GpuContext's startup self-test,
 * trellis2_mojo/gpu/context.mojo:7-12, 139-158): a small compute check plus
 * a wait on a device barrier that nothing completes, bounded to wait_us
 * microseconds (1..1e6). T2SC_OK when the compute is right and the bounded
 * wait came back with its timeout flag (the mechanism every conv pipeline
 * wait relies on); the context stays usable either way. */
int t2sc_ctx_selftest(t2sc_ctx *ctx, int wait_us);
/* Library version string, e.g. "t2sc 0.1 sm_100a". */
const char *t2sc_version(void);

/* ---- coordinates: device copy + coordinate hash + cached neighbour maps.
 * Equivalent of a SparseTensor's coords and its spatial cache
 * (sparse/basic.mojo:542-558): maps are built on first use per
 * (kernel, dilation) and reused by every conv on the same coordinates. ---- */
int t2sc_coords_create(t2sc_ctx *ctx, const int32_t *coords_host, int64_t n, t2sc_coords **out);
int t2sc_coords_create_device(t2sc_ctx *ctx, const int32_t *coords_dev, int64_t n, t2sc_coords **out);
/* Coordinates with halo rows (z-slab partition): rows [0, n_targets) are
 * this rank's own voxels and receive conv outputs; rows [n_targets, n) are
 * neighbours' boundary voxels that only act as sources. Conv inputs then
 * have n rows and outputs n_targets rows. on_device: coords is a device
 * pointer. New interface (the reference has no partitioned path). */
int t2sc_coords_create_halo(t2sc_ctx *ctx, const int32_t *coords, int64_t n, int64_t n_targets,
                            int on_device, t2sc_coords **out);
/* General form: target rows are [target_begin, target_end) of the n rows;
 * every row is a source. Conv outputs (and residuals) are indexed by target
 * row - target_begin, so a caller that keeps one [n, C] output buffer
 * passes y + target_begin * C. Exported edge lists use the same target
 * numbering. Lets a rank convolve its interior rows while the halo of its
 * boundary rows is still in flight. New interface (no reference counterpart). */
int t2sc_coords_create_range(t2sc_ctx *ctx, const int32_t *coords, int64_t n, int64_t target_begin,
                             int64_t target_end, int on_device, t2sc_coords **out);
int t2sc_coords_destroy(t2sc_coords *c);
/* Number of target rows (= all rows unless created with halo rows). */
int t2sc_coords_count(const t2sc_coords *c, int64_t *n);
/* Build (or fetch) the neighbour map; returns the edge count E. */
int t2sc_coords_build_map(t2sc_coords *c, int kd, int kh, int kw, int dilation, int64_t *n_edges);

/* Edge lists exactly as SparseConv3d._neighbor_map returns them
 * (conv.mojo:56-96): kernel-offset-major, target ascending. Host buffers of
 * capacity `cap`; if E > cap, returns T2SC_ERR_CAPACITY with *n_edges = E. */
int t2sc_neighbor_map_export(t2sc_coords *c, int kd, int kh, int kw, int dilation,
                             int64_t *src, int64_t *tgt, int64_t *kidx, int64_t cap,
                             int64_t *n_edges);
/* CSR exactly as conv.mojo:117-147 builds it: row_start [N+1], src_s [E],
 * kidx_s [E] (kernel index ascending within a row). */
int t2sc_csr_export(t2sc_coords *c, int kd, int kh, int kw, int dilation,
                    int64_t *row_start, int64_t *src_s, int64_t *kidx_s, int64_t cap,
                    int64_t *n_edges);

/* ---- conv: weights uploaded once (replaces GpuSparseConv.try_build,
 * gpu/conv.mojo:264-329). weight is host f32 [Co, Kd, Kh, Kw, Ci] (the
 * conv_none layout), bias host f32 [Co] or NULL. Unlike try_build there is
 * no Co % 64 gate and no decline: every shape runs on the GPU. The
 * reference's f16 weight storage (gpu/conv.mojo:32-36, chosen only when every
 * weight is f16-exact) needs no mode here: such weights are passed as f32
 * (exactly) and T2SC_DT_F32 gives the f32-storage result. ---- */
int t2sc_conv_create(t2sc_ctx *ctx, const float *weight, const float *bias, int co, int kd,
                     int kh, int kw, int ci, int dilation, int dtype, t2sc_conv **out);
int t2sc_conv_destroy(t2sc_conv *conv);

/* y [N, Co] = SubMConv(x [N, Ci]) + bias, then the epilogue flags.
 * Host f32 buffers in every dtype mode (16-bit modes round x to the mode's
 * type on the device). residual: host f32 [N, Co] or NULL. Replaces
 * SparseConv3d.forward (conv.mojo:98-199). */
int t2sc_conv_forward(t2sc_conv *conv, t2sc_coords *coords, const float *x, float *y, int flags,
                      const float *residual);
/* Same on device buffers whose element type is the conv's dtype (f32, f16
 * or bf16); asynchronous on the context stream. */
int t2sc_conv_forward_device(t2sc_conv *conv, t2sc_coords *coords, const void *x, void *y,
                             int flags, const void *residual);
/* A chain of convs on the same coordinates with device-resident
 * intermediates: host f32 x [N, Ci0] in, host f32 y [N, Co_last] out.
 * flags[i] applies to layer i; T2SC_RESIDUAL on layer i adds the chain input
 * x (the identity residual of a residual block). All convs share one dtype.
 * A set of >= 200k rows ordered by (batch, x) runs as x-slabs, each with a
 * halo as deep as the chain's reach along x, with slab uploads, convs and
 * downloads overlapped on the context's stream and two copy streams; the
 * results equal one unsplit pass. The slab plan (two coordinate handles
 * and maps per slab) is built on the first such call for a coordinate set
 * and kept with it; building it reads the coordinates back once. */
int t2sc_conv_chain_forward(t2sc_conv *const *convs, int n_layers, t2sc_coords *coords,
                            const float *x, float *y, const int *flags);

/* ---- subdivision (SparseUpsample / SparseChannel2Spatial
 * forward_subdivision). Children are emitted parent-major, child index
 * ascending; child c of parent (b,x,y,z) is (b, 2x + (c&1), 2y + ((c>>1)&1),
 * 2z + ((c>>2)&1)). Host buffers: sub f32 [N,8]; feats f32 [N,C] for
 * UPSAMPLE or [N,8*C] for C2S (C = output channels), NULL for NONE.
 * Outputs sized for the worst case M = 8N: out_coords int32 [8N,4],
 * out_feats f32 [8N,C], out_parent int64 [8N] (nullable),
 * out_subidx int64 [8N] (nullable). *m receives M. ---- */
int t2sc_subdivide(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub, int keep_mode,
                   const float *feats, int c, int feats_mode, int32_t *out_coords, float *out_feats,
                   int64_t *out_parent, int64_t *out_subidx, int64_t *m);
/* Device variant: feats/out_feats element type given by dtype; out_parent
 * and out_subidx are int32 on the device (nullable). *m is a host pointer;
 * the call synchronises the stream once to read it. */
int t2sc_subdivide_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub,
                          int keep_mode, const void *feats, int c, int feats_mode, int dtype,
                          int32_t *out_coords, void *out_feats, int32_t *out_parent,
                          int32_t *out_subidx, int64_t *m);

/* Allocation-free variant of t2sc_subdivide_device. It has no counterpart in
 * the reference; it exists for callers that may not allocate device memory
 * while they run (a runtime that hands the library a fixed memory budget up
 * front, or an engine that keeps the CUDA allocator and its implicit
 * synchronisation out of a decode pass). Its scratch (keep masks, counts,
 * offsets, scan block sums: about 13.6 MB) is one static device array per
 * GPU that loads the library, held until the process exits, sized for at
 * most 1,048,576 parents: a larger n is rejected with T2SC_ERR_INVALID and
 * a message. out_parent and out_subidx are required (int32 [8N] each).
 * The first call on a device looks up the array's device address; make
 * that first call before any stream capture. Every call on a device shares
 * the array, so calls that overlap on the GPU (other streams or contexts)
 * race; serialise them. Results are identical to t2sc_subdivide_device. */
int t2sc_subdivide_noalloc_device(t2sc_ctx *ctx, const int32_t *coords, int64_t n, const float *sub,
                                  int keep_mode, const void *feats, int c, int feats_mode, int dtype,
                                  int32_t *out_coords, void *out_feats, int32_t *out_parent,
                                  int32_t *out_subidx, int64_t *m);

/* ---- linear layers over feature rows ----
 * Replaces SparseLinear / linear (trellis2_mojo/modules/nn.mojo:27-266,
 * :268-293): y = x @ W^T + b, the ConvNeXt block's lin1 / lin2 and the
 * decoder's to_subdiv (models/sc_vaes/sparse_unet_vae.mojo:38-64, :79).
 * weight f32 [Co, Ci] host, bias f32 [Co] host (nullable); dtype as for
 * convs. The handle is a t2sc_conv with a 1x1x1 kernel (free it with
 * t2sc_conv_destroy) and runs on the same tcgen05 / CUDA-core kernels over
 * an identity row map, built (stream-ordered, without synchronising) on the
 * first call with a row count and kept on the context for every linear
 * layer; the first call with a new count should therefore come before any
 * stream capture. x device [rows, Ci], y device [rows, Co]
 * (must not alias x), flags T2SC_SILU / T2SC_RESIDUAL (residual [rows, Co])
 * fused into the epilogue, so lin2(silu(lin1(h))) + x is two calls. */
int t2sc_linear_create(t2sc_ctx *ctx, const float *weight, const float *bias, int co, int ci, int dtype,
                       t2sc_conv **out);
int t2sc_linear_forward_device(t2sc_conv *lin, const void *x, void *y, int64_t rows, int flags,
                               const void *residual);

/* ---- LayerNorm (+ SiLU) over the channel dim of device features ----
 * Replaces LayerNorm32.forward (trellis2_mojo/modules/nn.mojo:313-370) and,
 * with flags & T2SC_SILU, the activation(..., ACT_SILU) that follows it in
 * the decoder's upsample block (models/sc_vaes/sparse_unet_vae.mojo:118,123).
 * x, y: device [rows, c] of dtype (y may alias x); w, b: device f32 [c],
 * both NULL for affine=False. Per row: mean, population variance,
 * y = (x - mean) / sqrt(var + eps) (* w + b), then y / (1 + exp(-y)) for
 * SiLU; statistics in f32. 1 <= c <= 1024. Asynchronous on the stream. */
int t2sc_layernorm_device(t2sc_ctx *ctx, const void *x, void *y, int64_t rows, int c, const float *w,
                          const float *b, float eps, int flags, int dtype);

/* ---- the decoder's stage block: SparseConvNeXtBlock3d
 * (trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:40-64):
 *   y = lin2(SiLU(lin1(LN(conv(x))))) + x, LN affine eps 1e-6.
 * Weights host f32: conv [C,3,3,3,C] (+ bias [C]), norm w/b [C], lin1 [H,C]
 * (+ [H]), lin2 [C,H] (+ [C]). x, y: device [N, C] of dtype on `coords`
 * (no halo rows), y must not alias x. Asynchronous on the stream. */
typedef struct t2sc_convnext_block t2sc_convnext_block;
int t2sc_convnext_block_create(t2sc_ctx *ctx, int channels, int hidden, const float *conv_w, const float *conv_b,
                               const float *norm_w, const float *norm_b, const float *lin1_w, const float *lin1_b,
                               const float *lin2_w, const float *lin2_b, int dtype, t2sc_convnext_block **out);
int t2sc_convnext_block_destroy(t2sc_convnext_block *block);
int t2sc_convnext_block_forward_device(t2sc_convnext_block *block, t2sc_coords *coords, const void *x, void *y);

/* ---- the decoder's up block: SparseResBlockC2S3d
 * (trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:67-133):
 *   subdiv = to_subdiv(x) when pred_subdiv (Linear C -> 8), else given;
 *   h = conv1(SiLU(LN1(x)))            LN1 affine eps 1e-6, conv1 C -> 8*Cout;
 *   h = C2S(h, subdiv > 0); x2 = C2S(x, subdiv > 0)   (_binarize, :30-37);
 *   out = conv2(SiLU(LN2(h))) + repeat_interleave(x2, Cout / (C/8))
 *                                      LN2 no affine eps 1e-6, conv2 Cout -> Cout.
 * Weights host f32: norm1_w/b [C], conv1 [8*Cout,3,3,3,C] (+ bias [8*Cout]),
 * conv2 [Cout,3,3,3,Cout] (+ bias), to_subdiv [8,C] (+ bias [8]; NULL when
 * !pred_subdiv). C % 8 == 0, Cout a multiple of C/8, C and Cout <= 1024. */
typedef struct t2sc_c2s_block t2sc_c2s_block;
int t2sc_c2s_block_create(t2sc_ctx *ctx, int channels, int out_channels, int pred_subdiv, const float *norm1_w,
                          const float *norm1_b, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                          const float *conv2_b, const float *to_subdiv_w, const float *to_subdiv_b, int dtype,
                          t2sc_c2s_block **out);
int t2sc_c2s_block_destroy(t2sc_c2s_block *block);
/* forward (pred_subdiv: subdiv is an output, device f32 [N, 8]) and
 * forward_guided (!pred_subdiv: subdiv is the given device f32 [N, 8]).
 * x: device [N, C] of the block's dtype on `coords` (no halo rows);
 * out_coords: device int32 [8N, 4]; out_feats: device [8N, Cout] of the
 * dtype; *m (host) receives the child count M (the call synchronises once
 * to read it). out_child (nullable) receives a new coordinate handle of the
 * children with the conv2 map already built, owned by the caller. */
int t2sc_c2s_block_forward_device(t2sc_c2s_block *block, t2sc_coords *coords, const void *x, float *subdiv,
                                  int32_t *out_coords, void *out_feats, int64_t *m, t2sc_coords **out_child);

/* ---- multi-GPU data plane (no reference counterpart: the reference is
 * single-device, trellis2_mojo/gpu/context.mojo:116-165). One process per
 * GPU. A voxel set is cut into z-slabs of about equal voxel counts; each
 * rank convolves its own rows plus a halo of its z-neighbours' boundary
 * planes (t2sc_coords_create_halo with n_targets = counts[0]) and receives
 * that halo over NCCL before every layer. ---- */
#define T2SC_COMM_ID_BYTES 128
typedef struct t2sc_comm t2sc_comm;
/* The slab of `rank` among `world` (host code, every rank computes its
 * own). depth = dilation * (kernel / 2) (1 for the decoder's 3^3 convs);
 * every slab spans >= 2 * depth z planes (else T2SC_ERR_INVALID). rows
 * (capacity cap, NULL to query the counts) receives global row indices in
 * local order: interior own rows | own rows of the low band | own rows of
 * the high band | halo rows from rank - 1 | halo rows from rank + 1, each
 * group in global order. counts[6] = {own, interior, low band (sent to
 * rank - 1), high band (sent to rank + 1), halo from rank - 1, halo from
 * rank + 1}. */
int t2sc_partition_zslab(const int32_t *coords, int64_t n, int world, int rank, int depth, int64_t *rows,
                         int64_t cap, int64_t *counts);
/* A NCCL unique id (T2SC_COMM_ID_BYTES bytes) made by one rank and handed to
 * the others by the caller's own channel. T2SC_ERR_UNSUPPORTED when
 * libnccl.so.2 cannot be loaded. */
int t2sc_comm_unique_id(void *id_out);
/* Communicator of `nranks` processes on the context's device (NCCL loaded
 * at run time). Initialisation is polled and bounded by timeout_ms: a peer
 * that never joins gives T2SC_ERR_TIMEOUT and an aborted communicator. */
int t2sc_comm_create(t2sc_ctx *ctx, const void *id, int nranks, int rank, int timeout_ms, t2sc_comm **out);
/* Finalises (bounded) and frees the communicator. */
int t2sc_comm_destroy(t2sc_comm *comm);
/* Aborts the communicator's outstanding work (a peer failed). */
int t2sc_comm_abort(t2sc_comm *comm);
/* Fills the halo rows of device feats [own + halo rows, row_bytes] from the
 * z-neighbours: the low band goes to rank - 1 and the high band to rank + 1,
 * the halo arrives from both, as one grouped send/recv on the context's
 * stream (asynchronous; capturable in a CUDA graph). counts as returned by
 * t2sc_partition_zslab. */
int t2sc_halo_exchange_device(t2sc_comm *comm, void *feats, int64_t row_bytes, const int64_t *counts);
/* Waits for the context's stream, bounded by timeout_ms while polling the
 * communicator's asynchronous error state; on a timeout or a NCCL error
 * the communicator is aborted and T2SC_ERR_TIMEOUT / T2SC_ERR_CUDA returned. */
int t2sc_comm_wait(t2sc_comm *comm, int timeout_ms);

/* ---- pipeline glue around the decoder ----
 * FlexiDualGrid head: replaces fdg_head (trellis2_mojo/models/sc_vaes/
 * fdg_vae.mojo:17-50), the step of decode_shape (pipelines/image_to_3d.mojo:
 * 206-216) after the decoder. feats device f32 [t, 7]; outputs device f32:
 * vertices [t, 3] = (1 + 2*margin) * sigmoid(feats[:, 0:3]) - margin,
 * intersected [t, 3] = 1.0 where feats[:, 3:6] > 0 else 0.0, quad_lerp
 * [t, 1] = softplus(feats[:, 6]) (the value itself above 20). margin is
 * rounded to f32 as in the reference. Asynchronous on the stream. */
int t2sc_fdg_head_device(t2sc_ctx *ctx, const float *feats, int64_t t, double margin, float *vertices,
                         float *intersected, float *quad_lerp);

/* Cascade coordinates: replaces cascade_coords (trellis2_mojo/pipelines/
 * image_to_3d.mojo:219-270), called by run_cascade_stage
 * (run_image_to_3d.mojo:160-177) on the decoder's upsampled coordinates.
 * hr_coords device int32 [n, 4] (b, x, y, z), all >= 0. For hr_resolution =
 * resolution, resolution - 128, ...: q = int((xyz + 0.5) / lr_resolution *
 * (hr_resolution / 16)) in f32, rows (b, q) deduplicated and sorted
 * lexicographically; the first hr_resolution whose token count is below
 * max_num_tokens, or 1024, is taken. out_coords device int32 [n, 4]
 * receives *num_tokens rows; *hr_resolution (host) the resolution used.
 * Synchronises the stream twice per tried resolution. Where the reference
 * would loop without end (the budget never met and 1024 never reached)
 * this returns T2SC_ERR_INVALID once hr_resolution / 16 reaches 0;
 * max_num_tokens must be > 0; negative coordinates give T2SC_ERR_RANGE. */
int t2sc_cascade_coords_device(t2sc_ctx *ctx, const int32_t *hr_coords, int64_t n, int lr_resolution,
                               int resolution, int64_t max_num_tokens, int32_t *out_coords,
                               int64_t *num_tokens, int *hr_resolution);

/* Trilinear sampler: replaces grid_sample_trilinear (trellis2_mojo/meshing/
 * vertex_attrs.mojo:46-104; flex_gemm grid_sample_3d, mode trilinear, B = 1)
 * over the coordinate handle's own hash (rows of batch 0; a repeated voxel
 * resolves to its last row, as the reference's dictionary does). feats
 * device f32 [n, c] in the handle's row order; query device f32 [l, 3] in
 * voxel units; out device f32 [l, c]. The 8 neighbours of p are p +- 0.5
 * truncated toward zero; each weighs prod(1 - |n + 0.5 - p|); voxels absent,
 * negative or >= grid_size weigh 0; the sum is divided by max(weight sum,
 * 1e-12). grid_size <= 1536 (the hash's coordinate range). Asynchronous. */
int t2sc_grid_sample_trilinear_device(t2sc_coords *coords, const float *feats, int c, int grid_size,
                                      const float *query, int64_t l, float *out);

/* ---- synthetic inputs (seeded shells of the benchmark configurations) ----
 * Active cells of a G^3 grid with | |p-c| - R(1 + 0.1 sin(3t) cos(2(f+phase))) | <= h,
 * c = G/2, t = acos((p_z-c)/|p-c|), f = atan2(p_y-c, p_x-c), phase = 0 for
 * seed 0 else 2*pi*u0 (u0 = first draw of the project RNG, rng.mojo:20-37).
 * Rows lexicographic (b=batch, x, y, z). cap rows; *n receives the count. */
int t2sc_synth_shell(int g, double radius, double half_width, uint64_t seed, int batch,
                     int32_t *coords, int64_t cap, int64_t *n);
/* Standard normals * std from the project RNG (xorshift64* seeded by
 * splitmix64, Box-Muller; trellis2_mojo/rng.mojo:17-52). */
int t2sc_synth_normal(uint64_t seed, float std, float *out, int64_t count);
/* out[i] = 1.0 if next_f64() < p else 0.0 (seeded Bernoulli child mask). */
int t2sc_synth_bernoulli(uint64_t seed, double p, float *out, int64_t count);

#ifdef __cplusplus
}
#endif
#endif /* T2SC_H */
