/* CPU restatement of the TRELLIS.2-Mojo sparse submanifold-conv path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA
 * library (libt2sc) and the timed CPU baseline in bench.py. No product code
 * path loads it. Parity status: the algorithm follows the reference source
 * line by line (citations below); the reference is Mojo for osx-arm64 and
 * cannot run here, and its tests hold no stored outputs, so value-level
 * parity is UNPINNED. What is pinned: neighbour-edge counts for dense blobs
 * against the reference's published benchmark table
 * (docs/benchmarks/RESULTS.md:363-365: N=12,167 -> E=300,763;
 * N=54,872 -> E=1,404,928; N=216,000 -> E=5,639,752).
 */
#ifndef T2SC_ORACLE_H
#define T2SC_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Packed coordinate key, trellis2_mojo/sparse/conv.mojo:68-69 and :86-87. */
int64_t orc_pack_key(int64_t b, int64_t x, int64_t y, int64_t z);

/* Neighbour edge lists in the reference order (kernel-offset-major, target
 * ascending), trellis2_mojo/sparse/conv.mojo:56-96. Returns E. When E > cap
 * only the count is returned (outputs untouched beyond cap). */
int64_t orc_neighbor_map(const int32_t *coords, int64_t n, int kd, int kh,
                         int kw, int dilation, int64_t *src, int64_t *tgt,
                         int64_t *kidx, int64_t cap);

/* Stable counting sort of the edges by target, conv.mojo:117-147. */
void orc_csr(int64_t n, int64_t e, const int64_t *src, const int64_t *tgt,
             const int64_t *kidx, int64_t *row_start, int64_t *src_s,
             int64_t *kidx_s);

/* CPU SubM conv, conv.mojo:149-199. weight [Co, K, Ci] (= [Co,Kd,Kh,Kw,Ci]),
 * bias nullable. out [N, Co] is overwritten. nthreads <= 0: the reference's
 * own parallelism (chunks of 8 output channels, conv.mojo:166-194, as many
 * threads as chunks); nthreads > 0: that many threads over the same chunks. */
void orc_conv_forward(const float *x, int64_t n, int ci, const float *weight,
                      const float *bias, int co, int ksize, const int64_t *src,
                      const int64_t *tgt, const int64_t *kidx, int64_t e,
                      float *out, int nthreads);

/* All-cores variant: output rows split across threads, per-row edges walked
 * from the CSR (kidx ascending, the order conv.mojo:174 visits them for one
 * target), so each out[t,o] sums in exactly the reference order. */
void orc_conv_forward_rows(const float *x, int64_t n, int ci,
                           const float *weight, const float *bias, int co,
                           int ksize, const int64_t *row_start,
                           const int64_t *src_s, const int64_t *kidx_s,
                           float *out, int nthreads);

/* SiLU v/(1+exp(-v)), trellis2_mojo/modules/nn.mojo:567-568, in place. */
void orc_silu(float *v, int64_t n);
/* a += b (SparseTensor __add__, sparse/basic.mojo:438-439). */
void orc_add(float *a, const float *b, int64_t n);
/* Round every value to bf16 (mode 2) or f16 (mode 1), round-to-nearest-even. */
void orc_round16(float *v, int64_t n, int mode);

/* y = x @ W^T (+ b) (linear, trellis2_mojo/modules/nn.mojo:27-266): each
 * output a plain sequential f32 sum over k (the packed-GEMM order the
 * reference documents at nn.mojo:38-44), then optional SiLU and residual
 * (the epilogue order of the conv). w [co, ci], b nullable, res nullable. */
void orc_linear(const float *x, int64_t rows, int ci, const float *w, const float *b, int co, int silu,
                const float *res, float *out);

/* LayerNorm over the last dim (LayerNorm32.forward,
 * trellis2_mojo/modules/nn.mojo:313-370): 8-lane partial sums + halving-tree
 * reduce + scalar tail for the mean and the population variance,
 * inv_std = 1/sqrt(var + eps), optional affine (w, b nullable), then
 * optional SiLU (silu != 0; the decoder's norm -> activation pairs,
 * models/sc_vaes/sparse_unet_vae.mojo:118,123). */
void orc_layernorm(const float *x, int64_t rows, int c, const float *w, const float *b, float eps, int silu,
                   float *out);

/* Subdivision child list, sparse/spatial/basic.mojo:144-167 and
 * spatial/spatial2channel.mojo:97-116. positive=0: keep sub != 0 (the
 * forward_subdivision test); positive=1: keep sub > 0 (the decoder's
 * _binarize, models/sc_vaes/sparse_unet_vae.mojo:30-37). Returns M. */
int64_t orc_subdivide(const int32_t *coords, int64_t n, const float *sub,
                      int positive, int64_t *idx, int64_t *subidx,
                      int32_t *new_coords);
/* Upsample feats: out[e] = x[idx[e]] (spatial/basic.mojo:168). */
void orc_select_rows(const float *x, int c, const int64_t *idx, int64_t m,
                     float *out);
/* C2S unfold: out[e] = x[idx[e], subidx[e]*cout : +cout]
 * (spatial2channel.mojo:127-136). */
void orc_c2s_unfold(const float *x, int cout, const int64_t *idx,
                    const int64_t *subidx, int64_t m, float *out);

/* Seeded inputs (tests and the CPU reference of bench.py): the shell of
 * the benchmark configurations and the project RNG (rng.mojo:17-52). */
int64_t orc_synth_shell(int g, double radius, double h, uint64_t seed, int batch, int32_t *coords, int64_t cap);
void orc_synth_normal(uint64_t seed, float std_, float *out, int64_t count);
void orc_synth_bernoulli(uint64_t seed, double p, float *out, int64_t count);

/* Pipeline glue: fdg_head (models/sc_vaes/fdg_vae.mojo:17-50),
 * grid_sample_trilinear (meshing/vertex_attrs.mojo:46-104, xyz int32 [n,3]),
 * cascade_coords (pipelines/image_to_3d.mojo:219-270, hr int32 [n,4], out
 * [n,4]; returns the token count, -2 where the reference never ends). */
void orc_fdg_head(const float *f, int64_t t, double margin, float *vert, float *inter, float *quad);
int orc_grid_sample_trilinear(const float *feats, int64_t n, int c, const int32_t *xyz, int grid, const float *query,
                              int64_t l, float *out);
int64_t orc_cascade_coords(const int32_t *hr, int64_t n, int lr_res, int resolution, int64_t max_tokens,
                           int32_t *out, int *hr_out);

#ifdef __cplusplus
}
#endif
#endif
