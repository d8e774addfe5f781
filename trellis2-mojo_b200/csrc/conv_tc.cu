// Submanifold conv as an output-stationary gathered implicit GEMM on the
// sm_100a tensor cores (tcgen05, accumulators in TMEM).
//
// For an output tile of 128 rows (rows in neighbour-mask order, see
// hashmap.cu) and a tile of `bn` output channels:
//   D[128, bn] = sum over active offsets k, over Ci chunks c:
//                gather(x, nbr_sorted[k][tile rows])[128, chunk] * W[k][bn, chunk]^T
// Missing neighbours are zero-filled by the gather, so every output row is
// produced by exactly one CTA with no atomics. The tile only visits offsets
// set in its occupancy mask.
//
// Warp roles in a 288-thread CTA (persistent, one per SM):
//   warps 0-3  gather producers: cp.async 16-byte vectors of neighbour rows
//              into a 128B/64B/32B-swizzled K-major A stage; thread 0 also
//              bulk-copies the pre-swizzled weight block (B stage);
//   warps 4-7  epilogue: tcgen05.ld from TMEM, + bias, SiLU, + residual,
//              convert, store to the row's original position;
//   warp 8     TMEM owner and MMA issuer (one elected lane).
// Double-buffered TMEM accumulators let the epilogue of tile i overlap the
// MMAs of tile i+1. Every mbarrier wait is bounded; on timeout the CTA sets
// an error bit, drains its copies, frees TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "sm100.cuh"

namespace t2sc {
namespace {

constexpr int kProducerThreads = 128;
constexpr int kEpilogueThreads = 128;
constexpr int kThreads = kProducerThreads + kEpilogueThreads + 32;
constexpr int kLag = 2;                       // cp.async groups kept in flight per producer thread
constexpr long long kWaitLimit = 4000000000LL;  // ~2 s of SM clocks
constexpr int kSmemBudget = 200 * 1024;

struct TcArgs {
  const uint8_t *x;          // [n, ci] 16-bit
  uint8_t *y;                // [n, co] 16-bit
  const uint8_t *res;        // [n, co] 16-bit or null
  const uint8_t *wimg;       // pre-swizzled B blocks
  const float *bias;         // [co]
  const int32_t *nbr_sorted; // [K][n_pad]
  const int32_t *perm;       // [n_pad]
  const uint32_t *tile_mask; // [ntiles]
  int64_t n_pad;
  int ntiles, ci, co, bn, nchunks, nco_tiles, kvol, stages, flags, tmem_cols;
  uint32_t a_bytes, b_bytes, stage_bytes;
  int *err;
};

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (DT == T2SC_DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
}
template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if (DT == T2SC_DT_BF16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&v);
    return __bfloat1622float2(h);
  } else {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
  }
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// Epilogue for 16 consecutive output channels of one row.
template <int DT>
__device__ __forceinline__ void store16(const TcArgs &a, int orow, int col, const float (&acc)[16]) {
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = acc[i] + __ldg(a.bias + col + i);
  if (a.flags & T2SC_SILU) {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = silu(v[i]);
  }
  const int64_t off = ((int64_t)orow * a.co + col) * 2;
  if (a.flags & T2SC_RESIDUAL) {
    const uint4 *rp = reinterpret_cast<const uint4 *>(a.res + off);
    uint4 r0 = __ldg(rp), r1 = __ldg(rp + 1);
    uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float2 f = unpack2<DT>(rr[i]);
      v[2 * i] += f.x;
      v[2 * i + 1] += f.y;
    }
  }
  uint4 o0, o1;
  o0.x = pack2<DT>(v[0], v[1]);
  o0.y = pack2<DT>(v[2], v[3]);
  o0.z = pack2<DT>(v[4], v[5]);
  o0.w = pack2<DT>(v[6], v[7]);
  o1.x = pack2<DT>(v[8], v[9]);
  o1.y = pack2<DT>(v[10], v[11]);
  o1.z = pack2<DT>(v[12], v[13]);
  o1.w = pack2<DT>(v[14], v[15]);
  uint4 *yp = reinterpret_cast<uint4 *>(a.y + off);
  yp[0] = o0;
  yp[1] = o1;
}

// Warp-uniform bounded wait: lane 0 polls, the verdict is broadcast.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort, int *err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = sm100::mbar_wait_bounded(bar, parity, abort, err, kDevErrTimeout, kWaitLimit);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int DT, int RB>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)S * a.stage_bytes);
  // bars: full[S], empty[S], tfull[2], tempty[2], mma_done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 5);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const uint32_t sbase = sm100::smem_u32(smem);
  const uint32_t full0 = sm100::smem_u32(bars), empty0 = full0 + 8 * S;
  const uint32_t tfull0 = empty0 + 8 * S, tempty0 = tfull0 + 16, mma_done = tempty0 + 16;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      sm100::mbar_init(full0 + 8 * s, kProducerThreads + 1);
      sm100::mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; b++) {
      sm100::mbar_init(tfull0 + 8 * b, 1);
      sm100::mbar_init(tempty0 + 8 * b, kEpilogueThreads);
    }
    sm100::mbar_init(mma_done, 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 8) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), a.tmem_cols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nunits = a.ntiles * a.nco_tiles;
  constexpr int BKE = RB / 2;      // 16-bit elements per chunk row
  constexpr int CPR = RB / 16;     // 16-byte vectors per row
  constexpr int RPP = 32 / CPR;    // rows per warp pass

  if (warp < 4) {
    // ------------------------- gather producers -------------------------
    const int j = lane % CPR, rsub = lane / CPR;
    uint32_t it = 0;
    int npend = 0;
    uint32_t pend[kLag + 1];
    bool ok = true;
    for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const int tile = u / a.nco_tiles, cot = u % a.nco_tiles;
      uint32_t km = __ldg(a.tile_mask + tile);
      while (km && ok) {
        const int k = __ffs(km) - 1;
        km &= km - 1;
        int32_t srcs[CPR];
#pragma unroll
        for (int p = 0; p < CPR; p++) {
          const int row = 32 * warp + p * RPP + rsub;
          srcs[p] = __ldg(a.nbr_sorted + (int64_t)k * a.n_pad + (int64_t)tile * kTileRows + row);
        }
        for (int c = 0; c < a.nchunks; c++, it++) {
          const uint32_t s = it % S;
          if (!warp_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1, abort, a.err)) {
            ok = false;
            break;
          }
          const uint32_t abase = sbase + s * a.stage_bytes;
          if (tid == 0) {
            const uint32_t bbar = full0 + 8 * s;
            sm100::mbar_arrive_expect_tx(bbar, a.b_bytes);
            const uint8_t *wsrc = a.wimg + ((size_t)((size_t)cot * a.kvol + k) * a.nchunks + c) * a.b_bytes;
            sm100::bulk_g2s(abase + a.a_bytes, wsrc, a.b_bytes, bbar);
          }
          const int e0 = c * BKE + j * 8;
#pragma unroll
          for (int p = 0; p < CPR; p++) {
            const int row = 32 * warp + p * RPP + rsub;
            const int32_t src = srcs[p];
            const bool valid = src >= 0 && e0 < a.ci;
            const uint8_t *g = valid ? a.x + ((int64_t)src * a.ci + e0) * 2 : a.x;
            sm100::cp_async_16(abase + swizzle_off(row * RB + j * 16, RB), g, valid ? 16u : 0u);
          }
          sm100::cp_async_commit();
          pend[npend++] = s;
          if (npend > kLag) {
            sm100::cp_async_wait<kLag>();
            sm100::fence_proxy_async_smem();
            sm100::mbar_arrive(full0 + 8 * pend[0]);
            for (int q = 0; q < kLag; q++) pend[q] = pend[q + 1];
            npend--;
          }
        }
      }
    }
    sm100::cp_async_wait<0>();
    sm100::fence_proxy_async_smem();
    for (int q = 0; q < npend; q++) sm100::mbar_arrive(full0 + 8 * pend[q]);
    if (tid == 0 && !ok) {
      // let the weight bulk copies still in flight land before the CTA exits
      const uint32_t first = it > (uint32_t)S ? it - S : 0;
      for (uint32_t i2 = first; i2 < it; i2++)
        sm100::mbar_wait_cycles(full0 + 8 * (i2 % S), (i2 / S) & 1, kWaitLimit / 8);
    }
  } else if (warp < 8) {
    // ------------------------------ epilogue ------------------------------
    const int q = warp - 4;  // TMEM lane quadrant
    const int row = 32 * q + lane;
    uint32_t acc_it = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int tile = u / a.nco_tiles, cot = u % a.nco_tiles;
      const uint32_t km = __ldg(a.tile_mask + tile);
      const int orow = __ldg(a.perm + (int64_t)tile * kTileRows + row);
      const int col0 = cot * a.bn;
      if (km == 0) {
        if (orow >= 0) {
          float z[16];
#pragma unroll
          for (int i = 0; i < 16; i++) z[i] = 0.f;
          for (int cc = 0; cc < a.bn; cc += 16) store16<DT>(a, orow, col0 + cc, z);
        }
        continue;
      }
      const uint32_t b = acc_it & 1;
      if (!warp_wait(tfull0 + 8 * b, (acc_it >> 1) & 1, abort, a.err)) break;
      sm100::tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + b * a.bn;
      for (int cc = 0; cc < a.bn; cc += 16) {
        uint32_t r[16];
        sm100::tmem_ld16(tbase + cc, r);
        sm100::tmem_ld_wait();
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; i++) acc[i] = __uint_as_float(r[i]);
        if (orow >= 0) store16<DT>(a, orow, col0 + cc, acc);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(tempty0 + 8 * b);
      acc_it++;
    }
  } else {
    // ----------------------------- MMA issuer -----------------------------
    if (lane == 0) {
      const uint32_t idesc = sm100::instr_desc(DT == T2SC_DT_BF16 ? 1u : 0u, (uint32_t)a.bn);
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const int tile = u / a.nco_tiles;
        uint32_t km = __ldg(a.tile_mask + tile);
        if (km == 0) continue;
        const uint32_t b = acc_it & 1;
        if (!sm100::mbar_wait_bounded(tempty0 + 8 * b, ((acc_it >> 1) & 1) ^ 1, abort, a.err, kDevErrTimeout,
                                      kWaitLimit))
          break;
        sm100::tc_fence_after();
        const uint32_t dtm = tmem + b * a.bn;
        uint32_t accum = 0;
        const int nsteps = __popc(km) * a.nchunks;
        for (int st = 0; st < nsteps; st++, it++) {
          const uint32_t s = it % S;
          if (!sm100::mbar_wait_bounded(full0 + 8 * s, (it / S) & 1, abort, a.err, kDevErrTimeout, kWaitLimit)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t abase = sbase + s * a.stage_bytes, bbase = abase + a.a_bytes;
#pragma unroll
          for (int kk = 0; kk < RB / 32; kk++) {
            sm100::mma_f16(dtm, sm100::smem_desc(abase + kk * 32, RB), sm100::smem_desc(bbase + kk * 32, RB), idesc,
                           accum);
            accum = 1;
          }
          sm100::mma_commit(empty0 + 8 * s);
        }
        if (!ok) break;
        sm100::mma_commit(tfull0 + 8 * b);
        acc_it++;
      }
      // all issued MMAs retire before TMEM is released
      sm100::mma_commit(mma_done);
      sm100::mbar_wait_cycles(mma_done, 0, kWaitLimit / 8);
    }
    __syncwarp();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, a.tmem_cols);
  }
}

template <int DT, int RB>
int launch_tc(t2sc_conv *cv, const TcArgs &args, int grid, size_t smem, std::string &err) {
  auto kfn = conv_tc_kernel<DT, RB>;
  T2SC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "tc smem attr");
  kfn<<<grid, kThreads, smem, cv->ctx->stream>>>(args);
  T2SC_LAUNCHED(cv->ctx, "conv_tc");
  return T2SC_OK;
}

}  // namespace

// Chooses the tile shape and builds the pre-swizzled weight image: one
// block per (co tile, k, ci chunk) holding bn rows (output channels) x
// row_bytes (a chunk of input channels), exactly the B stage's smem image.
int conv_tc_prepare(t2sc_conv *cv, const float *w, std::string &err) {
  const int co = cv->co, ci = cv->ci, K = cv->kvol;
  cv->row_bytes = ci >= 64 ? 128 : (ci > 16 ? 64 : 32);
  const int bke = cv->row_bytes / 2;
  cv->nchunks = (ci + bke - 1) / bke;
  int bn = 0;
  for (int d = 256; d >= 16; d -= 16)
    if (co % d == 0) {
      bn = d;
      break;
    }
  cv->bn = bn;
  cv->nco_tiles = co / bn;
  const size_t bbytes = (size_t)bn * cv->row_bytes;
  const size_t total = bbytes * cv->nco_tiles * K * cv->nchunks;
  std::vector<uint16_t> img(total / 2, 0);
  for (int nt = 0; nt < cv->nco_tiles; nt++)
    for (int k = 0; k < K; k++)
      for (int c = 0; c < cv->nchunks; c++) {
        uint8_t *blk = reinterpret_cast<uint8_t *>(img.data()) + ((size_t)(nt * K + k) * cv->nchunks + c) * bbytes;
        for (int r = 0; r < bn; r++)
          for (int e = 0; e < bke; e++) {
            const int o = nt * bn + r, i = c * bke + e;
            float v = (i < ci) ? w[((size_t)o * K + k) * ci + i] : 0.0f;
            uint16_t bits;
            if (cv->dtype == T2SC_DT_BF16) {
              __nv_bfloat16 h = __float2bfloat16_rn(v);
              bits = *reinterpret_cast<uint16_t *>(&h);
            } else {
              __half h = __float2half_rn(v);
              bits = *reinterpret_cast<uint16_t *>(&h);
            }
            const uint32_t off = swizzle_off((uint32_t)(r * cv->row_bytes + e * 2), cv->row_bytes);
            *reinterpret_cast<uint16_t *>(blk + off) = bits;
          }
      }
  T2SC_CUDA(cudaMalloc(&cv->d_wtc, total), "conv weights");
  T2SC_CUDA(cudaMemcpy(cv->d_wtc, img.data(), total, cudaMemcpyHostToDevice), "conv weights upload");
  return T2SC_OK;
}

int conv_tc_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags, const void *residual,
                   std::string &err) {
  if (m->n == 0) return T2SC_OK;
  TcArgs a;
  a.x = static_cast<const uint8_t *>(x);
  a.y = static_cast<uint8_t *>(y);
  a.res = static_cast<const uint8_t *>(residual);
  a.wimg = static_cast<const uint8_t *>(cv->d_wtc);
  a.bias = cv->d_bias;
  a.nbr_sorted = m->nbr_sorted;
  a.perm = m->perm;
  a.tile_mask = m->tile_mask;
  a.n_pad = m->n_pad;
  a.ntiles = (int)m->ntiles;
  a.ci = cv->ci;
  a.co = cv->co;
  a.bn = cv->bn;
  a.nchunks = cv->nchunks;
  a.nco_tiles = cv->nco_tiles;
  a.kvol = cv->kvol;
  a.flags = flags;
  a.err = cv->ctx->d_err;
  int cols = 32;
  while (cols < 2 * cv->bn) cols <<= 1;
  a.tmem_cols = cols;
  a.a_bytes = kTileRows * cv->row_bytes;
  a.b_bytes = (uint32_t)cv->bn * cv->row_bytes;
  a.stage_bytes = (a.a_bytes + a.b_bytes + 1023u) & ~1023u;
  int S = kSmemBudget / (int)a.stage_bytes;
  if (S > 8) S = 8;
  if (S < kLag + 1) {
    err = "conv tile does not fit shared memory";
    return T2SC_ERR_UNSUPPORTED;
  }
  a.stages = S;
  // stages + barriers/slots + alignment slack; never below 120 KB so that a
  // single CTA owns each SM (and its TMEM).
  size_t smem = (size_t)S * a.stage_bytes + 256 + 1024;
  if (smem < 120 * 1024) smem = 120 * 1024;
  const int64_t nunits = (int64_t)a.ntiles * a.nco_tiles;
  const int grid = (int)(nunits < cv->ctx->num_sms ? nunits : cv->ctx->num_sms);
  const bool bf = cv->dtype == T2SC_DT_BF16;
  switch (cv->row_bytes) {
    case 128:
      return bf ? launch_tc<T2SC_DT_BF16, 128>(cv, a, grid, smem, err)
                : launch_tc<T2SC_DT_F16, 128>(cv, a, grid, smem, err);
    case 64:
      return bf ? launch_tc<T2SC_DT_BF16, 64>(cv, a, grid, smem, err)
                : launch_tc<T2SC_DT_F16, 64>(cv, a, grid, smem, err);
    default:
      return bf ? launch_tc<T2SC_DT_BF16, 32>(cv, a, grid, smem, err)
                : launch_tc<T2SC_DT_F16, 32>(cv, a, grid, smem, err);
  }
}

}  // namespace t2sc
