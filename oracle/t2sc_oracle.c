/* CPU restatement of the TRELLIS.2-Mojo sparse submanifold-conv path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libt2sc and the timed CPU
 * baseline of bench.py. Product code never loads it. Parity: follows the
 * reference source (cited per function); value-level parity is UNPINNED
 * (the Mojo reference cannot run here and its tests keep no outputs);
 * dense-blob edge counts are pinned to docs/benchmarks/RESULTS.md:363-365.
 *
 * Build: oracle/Makefile (gcc -O3 -pthread -ffp-contract=off). Floating
 * point contraction is off so every multiply and add rounds separately, as
 * the Mojo source writes them.
 */
#include "t2sc_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* Minimal parallel-for over [0, count) with a shared atomic cursor: each
 * thread takes `grain` items at a time. Stands in for Mojo's parallelize. */
typedef struct {
  void (*fn)(void *, int64_t, int64_t);
  void *arg;
  int64_t count, grain;
  int64_t next;
} pfor_t;
static void *pfor_worker(void *p) {
  pfor_t *job = (pfor_t *)p;
  for (;;) {
    int64_t lo = __atomic_fetch_add(&job->next, job->grain, __ATOMIC_RELAXED);
    if (lo >= job->count) break;
    int64_t hi = lo + job->grain < job->count ? lo + job->grain : job->count;
    job->fn(job->arg, lo, hi);
  }
  return NULL;
}
static void parallel_for(int nthreads, int64_t count, int64_t grain,
                         void (*fn)(void *, int64_t, int64_t), void *arg) {
  pfor_t job = {fn, arg, count, grain, 0};
  if (nthreads <= 1) { pfor_worker(&job); return; }
  pthread_t th[256];
  if (nthreads > 256) nthreads = 256;
  for (int i = 1; i < nthreads; i++) pthread_create(&th[i], NULL, pfor_worker, &job);
  pfor_worker(&job);
  for (int i = 1; i < nthreads; i++) pthread_join(th[i], NULL);
}

int64_t orc_pack_key(int64_t b, int64_t x, int64_t y, int64_t z) {
  /* conv.mojo:68-69: ((b*2048 + x + 512)*2048 + y + 512)*2048 + z + 512 */
  return ((b * 2048 + x + 512) * 2048 + y + 512) * 2048 + z + 512;
}

/* ---- a dictionary int64 -> row with Mojo Dict semantics (insert
 * overwrites, so the last row with a key wins: conv.mojo:67-70). ---- */
typedef struct {
  int64_t *keys;
  int64_t *vals;
  uint64_t mask;
} dict_t;

static uint64_t mix64(uint64_t k) {
  k ^= k >> 33; k *= 0xff51afd7ed558ccdULL;
  k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ULL;
  k ^= k >> 33; return k;
}
static void dict_init(dict_t *d, int64_t n) {
  uint64_t cap = 16;
  while (cap < (uint64_t)(2 * n + 1)) cap <<= 1;
  d->keys = (int64_t *)malloc(cap * sizeof(int64_t));
  d->vals = (int64_t *)malloc(cap * sizeof(int64_t));
  for (uint64_t i = 0; i < cap; i++) d->keys[i] = INT64_MIN;
  d->mask = cap - 1;
}
static void dict_put(dict_t *d, int64_t key, int64_t v) {
  uint64_t s = mix64((uint64_t)key) & d->mask;
  while (d->keys[s] != INT64_MIN && d->keys[s] != key) s = (s + 1) & d->mask;
  d->keys[s] = key;
  d->vals[s] = v;
}
static int64_t dict_get(const dict_t *d, int64_t key) {
  uint64_t s = mix64((uint64_t)key) & d->mask;
  while (d->keys[s] != INT64_MIN) {
    if (d->keys[s] == key) return d->vals[s];
    s = (s + 1) & d->mask;
  }
  return -1;
}
static void dict_free(dict_t *d) { free(d->keys); free(d->vals); }

int64_t orc_neighbor_map(const int32_t *coords, int64_t n, int kd, int kh,
                         int kw, int dilation, int64_t *src, int64_t *tgt,
                         int64_t *kidx, int64_t cap) {
  dict_t d;
  dict_init(&d, n);
  for (int64_t r = 0; r < n; r++) /* conv.mojo:67-70 */
    dict_put(&d, orc_pack_key(coords[4 * r], coords[4 * r + 1],
                              coords[4 * r + 2], coords[4 * r + 3]), r);
  int64_t e = 0;
  for (int kz = 0; kz < kd; kz++) /* conv.mojo:78-92 */
    for (int ky = 0; ky < kh; ky++)
      for (int kx = 0; kx < kw; kx++) {
        int64_t oz = (int64_t)(kz - kd / 2) * dilation; /* column 1 */
        int64_t oy = (int64_t)(ky - kh / 2) * dilation; /* column 2 */
        int64_t ox = (int64_t)(kx - kw / 2) * dilation; /* column 3 */
        int64_t k = (int64_t)kz * kh * kw + (int64_t)ky * kw + kx;
        for (int64_t r = 0; r < n; r++) {
          const int32_t *c = coords + 4 * r;
          int64_t key = orc_pack_key(c[0], (int64_t)c[1] + oz,
                                     (int64_t)c[2] + oy, (int64_t)c[3] + ox);
          int64_t hit = dict_get(&d, key);
          if (hit >= 0) {
            if (e < cap) { src[e] = hit; tgt[e] = r; kidx[e] = k; }
            e++;
          }
        }
      }
  dict_free(&d);
  return e;
}

void orc_csr(int64_t n, int64_t e, const int64_t *src, const int64_t *tgt,
             const int64_t *kidx, int64_t *row_start, int64_t *src_s,
             int64_t *kidx_s) {
  /* conv.mojo:125-141 */
  int64_t *cur = (int64_t *)calloc((size_t)n + 1, sizeof(int64_t));
  for (int64_t i = 0; i < e; i++) cur[tgt[i]]++;
  int64_t run = 0;
  for (int64_t r = 0; r < n; r++) { row_start[r] = run; run += cur[r]; }
  row_start[n] = run;
  for (int64_t r = 0; r < n; r++) cur[r] = row_start[r];
  for (int64_t i = 0; i < e; i++) {
    int64_t p = cur[tgt[i]]++;
    src_s[p] = src[i];
    kidx_s[p] = kidx[i];
  }
  free(cur);
}

/* One edge's dot over Ci: 8-lane partial sums (conv.mojo:179-183), the lane
 * reduce (SIMD.reduce_add, :184, restated as the halving tree
 * (l, l+4) -> (l, l+2) -> (0, 1)), then the scalar tail (:185-187). */
static inline float edge_dot(const float *xr, const float *wr, int ci) {
  float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= ci; i += 8)
    for (int l = 0; l < 8; l++) a[l] += xr[i + l] * wr[i + l];
  float t4[4], t2[2];
  for (int l = 0; l < 4; l++) t4[l] = a[l] + a[l + 4];
  for (int l = 0; l < 2; l++) t2[l] = t4[l] + t4[l + 2];
  float acc = t2[0] + t2[1];
  for (; i < ci; i++) acc += xr[i] * wr[i];
  return acc;
}

typedef struct {
  const float *x, *weight;
  int ci, co, ksize;
  const int64_t *src, *tgt, *kidx;
  int64_t e;
  float *out;
} chunk_args;
static void conv_chunks(void *p, int64_t lo, int64_t hi) {
  const chunk_args *a = (const chunk_args *)p;
  const int OCH = 8; /* conv.mojo:167 */
  for (int64_t wk = lo; wk < hi; wk++) { /* conv.mojo:171-188 */
    int o_lo = (int)wk * OCH, o_hi = o_lo + OCH < a->co ? o_lo + OCH : a->co;
    for (int64_t i = 0; i < a->e; i++) {
      const float *xr = a->x + a->src[i] * a->ci;
      float *orow = a->out + a->tgt[i] * a->co;
      for (int o = o_lo; o < o_hi; o++)
        orow[o] += edge_dot(xr, a->weight + ((int64_t)o * a->ksize + a->kidx[i]) * a->ci, a->ci);
    }
  }
}

void orc_conv_forward(const float *x, int64_t n, int ci, const float *weight,
                      const float *bias, int co, int ksize, const int64_t *src,
                      const int64_t *tgt, const int64_t *kidx, int64_t e,
                      float *out, int nthreads) {
  int n_work = (co + 7) / 8;
  memset(out, 0, sizeof(float) * (size_t)n * co);
  int nt = nthreads > 0 ? nthreads : n_work;
  chunk_args a = {x, weight, ci, co, ksize, src, tgt, kidx, e, out};
  parallel_for(nt, n_work, 1, conv_chunks, &a);
  if (bias) /* conv.mojo:195-198 */
    for (int64_t r = 0; r < n; r++)
      for (int o = 0; o < co; o++) out[r * co + o] += bias[o];
}

typedef struct {
  const float *x, *weight, *bias;
  int ci, co, ksize;
  const int64_t *row_start, *src_s, *kidx_s;
  float *out;
} rows_args;
static void conv_rows(void *p, int64_t lo, int64_t hi) {
  const rows_args *a = (const rows_args *)p;
  int co = a->co, ci = a->ci;
  for (int64_t t = lo; t < hi; t++) {
    float *orow = a->out + t * co;
    for (int o = 0; o < co; o++) orow[o] = 0.0f;
    for (int64_t q = a->row_start[t]; q < a->row_start[t + 1]; q++) {
      const float *xr = a->x + a->src_s[q] * ci;
      for (int o = 0; o < co; o++)
        orow[o] += edge_dot(xr, a->weight + ((int64_t)o * a->ksize + a->kidx_s[q]) * ci, ci);
    }
    if (a->bias)
      for (int o = 0; o < co; o++) orow[o] += a->bias[o];
  }
}

void orc_conv_forward_rows(const float *x, int64_t n, int ci,
                           const float *weight, const float *bias, int co,
                           int ksize, const int64_t *row_start,
                           const int64_t *src_s, const int64_t *kidx_s,
                           float *out, int nthreads) {
  rows_args a = {x, weight, bias, ci, co, ksize, row_start, src_s, kidx_s, out};
  parallel_for(nthreads > 0 ? nthreads : 1, n, 256, conv_rows, &a);
}

void orc_silu(float *v, int64_t n) {
  for (int64_t i = 0; i < n; i++) v[i] = v[i] / (1.0f + expf(-v[i]));
}

void orc_add(float *a, const float *b, int64_t n) {
  for (int64_t i = 0; i < n; i++) a[i] += b[i];
}

static float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan */
    if (u & 0x7fffffu) u |= 0x00400000u;
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  memcpy(&f, &u, 4);
  return f;
}
static float round_f16(float f) {
  /* round to the nearest f16 value (ties to even) via scaling: values in
   * the f16 normal range keep 11 significant bits; the subnormal range has
   * a fixed quantum of 2^-24. Saturates to inf beyond 65520. */
  float a = fabsf(f);
  if (!(a == a) || a == INFINITY) return f;
  if (a >= 65520.0f) return copysignf(INFINITY, f);
  int ex;
  frexpf(a, &ex); /* a = m * 2^ex, m in [0.5,1) */
  int q = ex - 11; /* quantum exponent for 11 significant bits */
  if (q < -24) q = -24;
  float scale = ldexpf(1.0f, -q);
  float r = nearbyintf(a * scale) / scale; /* default rounding: ties-to-even */
  return copysignf(r, f);
}
void orc_round16(float *v, int64_t n, int mode) {
  for (int64_t i = 0; i < n; i++) v[i] = mode == 2 ? round_bf16(v[i]) : round_f16(v[i]);
}

int64_t orc_subdivide(const int32_t *coords, int64_t n, const float *sub,
                      int positive, int64_t *idx, int64_t *subidx,
                      int32_t *new_coords) {
  int64_t m = 0;
  for (int64_t r = 0; r < n; r++) /* spatial/basic.mojo:156-160 */
    for (int c = 0; c < 8; c++) {
      float s = sub[r * 8 + c];
      int keep = positive ? (s > 0.0f) : (s != 0.0f);
      if (keep) {
        idx[m] = r;
        subidx[m] = c;
        m++;
      }
    }
  for (int64_t e = 0; e < m; e++) { /* spatial/basic.mojo:163-167 */
    const int32_t *p = coords + 4 * idx[e];
    int32_t *q = new_coords + 4 * e;
    q[0] = p[0];
    for (int i = 0; i < 3; i++) {
      int child = (int)(subidx[e] >> i) & 1; /* subidx // 2^i % 2 */
      q[i + 1] = p[i + 1] * 2 + child;
    }
  }
  return m;
}

void orc_select_rows(const float *x, int c, const int64_t *idx, int64_t m,
                     float *out) {
  for (int64_t e = 0; e < m; e++)
    memcpy(out + e * c, x + idx[e] * c, sizeof(float) * c);
}

void orc_c2s_unfold(const float *x, int cout, const int64_t *idx,
                    const int64_t *subidx, int64_t m, float *out) {
  for (int64_t e = 0; e < m; e++) { /* spatial2channel.mojo:133-136 */
    int64_t slot = idx[e] * 8 + subidx[e];
    memcpy(out + e * cout, x + slot * cout, sizeof(float) * cout);
  }
}

static float reduce8(const float *a) { /* SIMD.reduce_add as the halving tree */
  float t4[4], t2[2];
  for (int l = 0; l < 4; l++) t4[l] = a[l] + a[l + 4];
  for (int l = 0; l < 2; l++) t2[l] = t4[l] + t4[l + 2];
  return t2[0] + t2[1];
}

void orc_layernorm(const float *x, int64_t rows, int c, const float *w, const float *b, float eps, int silu,
                   float *out) {
  for (int64_t r = 0; r < rows; r++) { /* nn.mojo:324-369 */
    const float *xr = x + r * c;
    float *orow = out + r * c;
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= c; i += 8)
      for (int l = 0; l < 8; l++) s[l] += xr[i + l];
    float mean = reduce8(s);
    for (; i < c; i++) mean += xr[i];
    mean /= (float)c;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    i = 0;
    for (; i + 8 <= c; i += 8)
      for (int l = 0; l < 8; l++) {
        float d = xr[i + l] - mean;
        v[l] += d * d;
      }
    float var = reduce8(v);
    for (; i < c; i++) {
      float d = xr[i] - mean;
      var += d * d;
    }
    var /= (float)c;
    float inv_std = 1.0f / sqrtf(var + eps);
    for (i = 0; i < c; i++) {
      float y = (xr[i] - mean) * inv_std;
      if (w) y = y * w[i] + b[i];
      if (silu) y = y / (1.0f + expf(-y));
      orow[i] = y;
    }
  }
}

void orc_linear(const float *x, int64_t rows, int ci, const float *w, const float *b, int co, int silu,
                const float *res, float *out) {
  for (int64_t r = 0; r < rows; r++)
    for (int o = 0; o < co; o++) {
      float acc = 0.0f;
      for (int k = 0; k < ci; k++) acc += x[r * ci + k] * w[(int64_t)o * ci + k];
      if (b) acc += b[o];
      if (silu) acc = acc / (1.0f + expf(-acc));
      if (res) acc += res[r * co + o];
      out[r * co + o] = acc;
    }
}

/* ---- seeded inputs, restated independently of the product library so
 * that the timed CPU reference never loads libt2sc. The RNG is the
 * project's (trellis2_mojo/rng.mojo:17-52): splitmix64 seeding of an
 * xorshift64* stream, 53-bit uniforms, Box-Muller normals. ---- */
typedef struct { uint64_t s; } orc_rng;
static orc_rng rng_seed(uint64_t seed) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ULL; /* splitmix64 step */
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  z ^= z >> 31;
  orc_rng r = {z ? z : 0x9E3779B97F4A7C15ULL};
  return r;
}
static uint64_t rng_u64(orc_rng *r) { /* xorshift64* */
  r->s ^= r->s >> 12;
  r->s ^= r->s << 25;
  r->s ^= r->s >> 27;
  return r->s * 0x2545F4914F6CDD1DULL;
}
static double rng_f64(orc_rng *r) { return (double)(rng_u64(r) >> 11) / 9007199254740992.0; }

int64_t orc_synth_shell(int g, double radius, double h, uint64_t seed, int batch, int32_t *coords, int64_t cap) {
  const double two_pi = 6.283185307179586;
  double phase = 0.0;
  if (seed) {
    orc_rng r = rng_seed(seed);
    phase = two_pi * rng_f64(&r);
  }
  const double c = g / 2.0, lo = 0.9 * radius - h - 1.0, hi = 1.1 * radius + h + 1.0;
  int64_t m = 0;
  for (int x = 0; x < g; x++)
    for (int y = 0; y < g; y++)
      for (int z = 0; z < g; z++) {
        double dx = x - c, dy = y - c, dz = z - c;
        double rad = sqrt(dx * dx + dy * dy + dz * dz);
        if (rad < lo || rad > hi) continue; /* cannot be within h of the surface */
        double th = rad > 0 ? acos(dz / rad) : 0.0, ph = atan2(dy, dx) + phase;
        double surf = radius * (1.0 + 0.1 * sin(3.0 * th) * cos(2.0 * ph));
        if (fabs(rad - surf) > h) continue;
        if (coords && m < cap) {
          coords[4 * m] = batch;
          coords[4 * m + 1] = x;
          coords[4 * m + 2] = y;
          coords[4 * m + 3] = z;
        }
        m++;
      }
  return m;
}

void orc_synth_normal(uint64_t seed, float std_, float *out, int64_t count) {
  orc_rng r = rng_seed(seed);
  for (int64_t i = 0; i < count; i++) {
    double u1;
    do u1 = rng_f64(&r); while (u1 == 0.0);
    double u2 = rng_f64(&r);
    out[i] = (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2)) * std_;
  }
}

void orc_synth_bernoulli(uint64_t seed, double p, float *out, int64_t count) {
  orc_rng r = rng_seed(seed);
  for (int64_t i = 0; i < count; i++) out[i] = rng_f64(&r) < p ? 1.0f : 0.0f;
}

/* ---- pipeline glue around the decoder ---- */

/* fdg_head, trellis2_mojo/models/sc_vaes/fdg_vae.mojo:17-50: f32 arithmetic
 * with the reference's exp/log (libm expf/logf here). */
void orc_fdg_head(const float *f, int64_t t, double margin, float *vert, float *inter, float *quad) {
  const float m = (float)margin;
  for (int64_t r = 0; r < t; r++) {
    for (int c = 0; c < 3; c++) {
      const float x = f[r * 7 + c];
      vert[r * 3 + c] = (1.0f + 2.0f * m) / (1.0f + expf(-x)) - m;
    }
    for (int c = 0; c < 3; c++) inter[r * 3 + c] = f[r * 7 + 3 + c] > 0 ? 1.0f : 0.0f;
    const float q = f[r * 7 + 6];
    quad[r] = q > 20 ? q : logf(1.0f + expf(q));
  }
}

/* The sampler's voxel lookup keys rows by (x << 42) | (y << 21) | z
 * (vertex_attrs.mojo:40-43); rows are inserted in order with overwrite, so a
 * repeated voxel keeps its last row (Dict). */
/* grid_sample_trilinear, trellis2_mojo/meshing/vertex_attrs.mojo:46-104. */
int orc_grid_sample_trilinear(const float *feats, int64_t n, int c, const int32_t *xyz, int grid, const float *query,
                              int64_t l, float *out) {
  static const float off[24] = {-0.5f, -0.5f, -0.5f, -0.5f, -0.5f, 0.5f, -0.5f, 0.5f, -0.5f, -0.5f, 0.5f, 0.5f,
                                0.5f,  -0.5f, -0.5f, 0.5f,  -0.5f, 0.5f, 0.5f,  0.5f, -0.5f, 0.5f,  0.5f, 0.5f};
  dict_t d;
  dict_init(&d, n);
  float *acc = (float *)malloc((size_t)c * sizeof(float));
  if (!d.keys || !d.vals || !acc) { dict_free(&d); free(acc); return -1; }
  for (int64_t i = 0; i < n; i++)
    dict_put(&d, ((int64_t)xyz[3 * i] << 42) | ((int64_t)xyz[3 * i + 1] << 21) | (int64_t)xyz[3 * i + 2], i);
  for (int64_t q = 0; q < l; q++) {
    const float px = query[q * 3], py = query[q * 3 + 1], pz = query[q * 3 + 2];
    for (int ch = 0; ch < c; ch++) acc[ch] = 0;
    float wsum = 0;
    for (int k = 0; k < 8; k++) {
      const float fx = px + off[k * 3], fy = py + off[k * 3 + 1], fz = pz + off[k * 3 + 2];
      if (!(fx > -1.0f && fy > -1.0f && fz > -1.0f)) continue;  /* truncates to a negative index: miss */
      if (fx >= (float)grid || fy >= (float)grid || fz >= (float)grid) continue;
      const int64_t nx = (int64_t)fx, ny = (int64_t)fy, nz = (int64_t)fz;  /* toward zero */
      if (nx >= grid || ny >= grid || nz >= grid) continue;
      const int64_t idx = dict_get(&d, (nx << 42) | (ny << 21) | nz);
      if (idx < 0) continue;
      const float w = (1.0f - fabsf((float)nx + 0.5f - px)) * (1.0f - fabsf((float)ny + 0.5f - py)) *
                      (1.0f - fabsf((float)nz + 0.5f - pz));
      wsum += w;
      for (int ch = 0; ch < c; ch++) acc[ch] += w * feats[idx * c + ch];
    }
    const float denom = wsum < 1e-12f ? 1e-12f : wsum;
    for (int ch = 0; ch < c; ch++) out[q * c + ch] = acc[ch] / denom;
  }
  dict_free(&d);
  free(acc);
  return 0;
}

static int cmp_i64(const void *a, const void *b) {
  const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
  return x < y ? -1 : (x > y);
}

/* cascade_coords, trellis2_mojo/pipelines/image_to_3d.mojo:219-270. out
 * [n, 4]; returns the token count (-1: allocation failure, -2: the budget
 * is never met, where the reference would not terminate). */
int64_t orc_cascade_coords(const int32_t *hr, int64_t n, int lr_res, int resolution, int64_t max_tokens,
                           int32_t *out, int *hr_out) {
  int64_t *qs = (int64_t *)malloc((size_t)(3 * n + 1) * sizeof(int64_t));
  int64_t *keys = (int64_t *)malloc((size_t)(n + 1) * sizeof(int64_t));
  if (!qs || !keys) { free(qs); free(keys); return -1; }
  for (int hr_res = resolution;; hr_res -= 128) {
    const int k = hr_res / 16;
    if (k <= 0) { free(qs); free(keys); return -2; }
    int64_t qmax = 0;
    for (int64_t r = 0; r < n; r++)
      for (int c = 1; c < 4; c++) {
        const int64_t q = (int64_t)(((float)hr[r * 4 + c] + 0.5f) / (float)lr_res * (float)k);
        qs[r * 3 + c - 1] = q;
        if (q > qmax) qmax = q;
      }
    const int64_t m = qmax + 1;
    for (int64_t r = 0; r < n; r++) {
      int64_t key = hr[r * 4];
      for (int c = 0; c < 3; c++) key = key * m + qs[r * 3 + c];
      keys[r] = key;
    }
    qsort(keys, (size_t)n, sizeof(int64_t), cmp_i64);
    int64_t tokens = 0;
    for (int64_t i = 0; i < n; i++)
      if (i == 0 || keys[i] != keys[i - 1]) tokens++;
    if (tokens < max_tokens || hr_res == 1024) {
      int64_t e = 0;
      for (int64_t i = 0; i < n; i++) {
        if (i > 0 && keys[i] == keys[i - 1]) continue;
        int64_t key = keys[i];
        out[e * 4 + 3] = (int32_t)(key % m); key /= m;
        out[e * 4 + 2] = (int32_t)(key % m); key /= m;
        out[e * 4 + 1] = (int32_t)(key % m);
        out[e * 4 + 0] = (int32_t)(key / m);
        e++;
      }
      *hr_out = hr_res;
      free(qs); free(keys);
      return tokens;
    }
  }
}
