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
//   warps 0-3  epilogue: tcgen05.ld from TMEM, + bias, SiLU, + residual,
//              convert, store to the row's original position;
//   warps 4-7  gather producers: 16-byte cp.async vectors of the neighbour
//              rows straight into the 128B/64B/32B-swizzled K-major A tile
//              (zero-filled for a missing neighbour); each thread publishes
//              its copies with cp.async.mbarrier.arrive.noinc, so up to S
//              stages are in flight. Thread 0 of the group also bulk-copies
//              the pre-swizzled weight block (B tile) and prefetches each
//              tile's neighbour-index block into shared memory a tile ahead;
//   warp 8     TMEM owner and MMA issuer (the converged warp; elect.sync issues).
// Double-buffered TMEM accumulators let the epilogue of tile i overlap the
// MMAs of tile i+1.
//
// Modes: f16 / bf16 (kind::f16, one MMA per 16-wide k-step) and the
// f32-accurate split-TF32 mode (kind::tf32): x = x_hi + x_lo and
// w = w_hi + w_lo with x_hi, w_hi rounded to TF32, and
// D += x_hi*w_hi + x_hi*w_lo + x_lo*w_hi (the x_lo*w_lo term, ~2^-22
// relative, is dropped). The A stage then holds the hi and lo gathers, the
// B stage the hi and lo weight blocks. Because the tensor core's f32
// accumulation rounds (biased) at every step, this mode drains the TMEM
// accumulator after every kernel offset and sums the 27 partials in
// registers, which keeps the error near the f32 level.
//
// Every mbarrier wait is bounded; on timeout the CTA sets an error bit,
// lets its copies land, frees TMEM and returns.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "epilogue.cuh"
#include "sm100.cuh"

#ifndef T2SC_CONV_DIAGNOSTICS
#define T2SC_CONV_DIAGNOSTICS 0
#endif

// copy warps per CTA in the 16-bit modes: 4 measured ~10 % faster than 8 at
// the 512^3 decoder level (0.130 vs 0.145 ms per layer)
#ifndef T2SC_COPY_WARPS
#define T2SC_COPY_WARPS 4
#endif

namespace t2sc {
namespace {

constexpr int kEpilogueThreads = 128;
constexpr int kMinStages = 3;
constexpr int kTf32MaxBn = 128;                  // register-resident partial sums per row
constexpr long long kWaitLimit = 4000000000LL;  // ~2 s of SM clocks
constexpr int kSmemMax = 232448;  // 227 KB: the sm_100 per-block dynamic shared memory limit
constexpr int kSmemHalf = 115712;  // per block when two share an SM's 228 KB (1 KB reserved each)
#ifndef T2SC_CTAS_PER_SM
#define T2SC_CTAS_PER_SM 2
#endif
constexpr int kDefaultCtasPerSm = T2SC_CTAS_PER_SM;
constexpr int kModeTf32x3 = kEpiF32;  // beside T2SC_DT_F16 (1) and T2SC_DT_BF16 (2)
constexpr int kCopyWarp0 = 4;
// Warp roles: 0-3 epilogue; kCopyWarps copy warps (T2SC_COPY_WARPS in the
// 16-bit modes, 4 in the split-TF32 mode); one control warp (weight copies,
// index prefetch); one MMA warp.
template <int DT, int RB = 128>
struct Roles {
  // 16-byte vectors per row: each warp must own >= 32 / (RB / 16) rows
  static constexpr int kCopyWarps = DT == 3 ? 4 : T2SC_COPY_WARPS;
  static constexpr int kControlWarp = kCopyWarp0 + kCopyWarps;
  static constexpr int kMmaWarp = kControlWarp + 1;
  static constexpr int kThreads = 32 * (kMmaWarp + 1);
};

struct TcArgs {
  const uint8_t *x;          // [n_src, ci] 16-bit, or the f32 hi parts (split-TF32 mode)
  const uint8_t *x_lo;       // [n_src, ci] f32 lo parts (split-TF32 mode)
  uint8_t *y;                // [n, co] 16-bit or f32
  const uint8_t *res;        // [n, co] like y, or null
  const uint8_t *wimg;       // pre-swizzled B blocks
  const float *bias;         // [co]
  const int32_t *nbr_sorted; // [K][n_pad]
  const int32_t *perm;       // [n_pad]
  const uint32_t *tile_mask; // [ntiles]
  int64_t n_pad;
  int ntiles, ci, co, bn, nchunks, nco_tiles, kvol, stages, flags, tmem_cols;
  uint32_t a_bytes, b_bytes, sub_bytes, stage_bytes;  // per (k, chunk) pair: A, B; pair slot; stage
  int group;                                          // (k, chunk) pairs per pipeline stage
#if T2SC_CONV_DIAGNOSTICS
  int debug;  // diagnostics (T2SC_CONV_DEBUG): 1 skips the gathers, 2 the MMAs, 4 the epilogue stores
  long long *trace;  // diagnostics (T2SC_CONV_TRACE): per-stage clocks of CTA 0, or null
#endif
  int *err;
};
// Diagnostics build only (-DT2SC_CONV_DIAGNOSTICS=1, never the product
// library): switches that skip parts of the work and a per-stage clock trace.
#if T2SC_CONV_DIAGNOSTICS
constexpr int kTraceN = 4096;
#define T2SC_TRACE(slot, idx)                                                     \
  do {                                                                            \
    if (a.trace && blockIdx.x == 0 && (idx) < kTraceN) a.trace[(slot) * kTraceN + (idx)] = clock64(); \
  } while (0)
#define T2SC_SKIP(bit) (a.debug & (bit))
#else
#define T2SC_TRACE(slot, idx) \
  do {                        \
  } while (0)
#define T2SC_SKIP(bit) false
#endif

// Warp-uniform bounded wait: every lane probes the barrier (the common
// case, an already completed phase, costs one probe); a lane that has to
// wait falls into the bounded loop; the verdict is agreed with a vote.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort, int *err) {
  bool ok = sm100::mbar_test_wait(bar, parity);
  if (__all_sync(0xffffffffu, ok)) return true;
  if (!ok) ok = sm100::mbar_wait_bounded(bar, parity, abort, err, kDevErrTimeout, kWaitLimit);
  return __all_sync(0xffffffffu, ok);
}

template <int DT, int RB>
__global__ void __launch_bounds__(Roles<DT, RB>::kThreads, 1)
    conv_tc_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  // neighbour indices of a tile's active offsets, double-buffered across tiles
  int32_t *idx_buf = reinterpret_cast<int32_t *>(smem + (size_t)S * a.stage_bytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(idx_buf + 2 * kMaxK * kTileRows);
  // bars: full[S], empty[S], tfull[2], tempty[2], mma_done, idx_full[2], idx_empty[2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 9);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const uint32_t sbase = sm100::smem_u32(smem);
  const uint32_t full0 = sm100::smem_u32(bars), empty0 = full0 + 8 * S;
  const uint32_t tfull0 = empty0 + 8 * S, tempty0 = tfull0 + 16, mma_done = tempty0 + 16;
  const uint32_t idxf0 = mma_done + 8, idxe0 = idxf0 + 16;

  constexpr bool kSplit = DT == kModeTf32x3;
  constexpr int kW = Roles<DT, RB>::kCopyWarps, kControlWarp = Roles<DT, RB>::kControlWarp, kMmaWarp = Roles<DT, RB>::kMmaWarp;
  constexpr int ES = kSplit ? 4 : 2;   // element bytes
  constexpr int BKE = RB / ES;         // elements per chunk row
  const uint32_t a_tile = kTileRows * RB, b_tile = (uint32_t)a.bn * RB;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      // one cp.async completion arrival per copy lane + the control warp's expect_tx
      sm100::mbar_init(full0 + 8 * s, 32 * kW + 1);
      sm100::mbar_init(empty0 + 8 * s, 1);  // one tcgen05.commit
    }
    for (int b = 0; b < 2; b++) {
      sm100::mbar_init(tfull0 + 8 * b, 1);
      sm100::mbar_init(tempty0 + 8 * b, kEpilogueThreads / 32);  // one arrival per epilogue warp
    }
    sm100::mbar_init(mma_done, 1);
    for (int b = 0; b < 2; b++) {
      sm100::mbar_init(idxf0 + 8 * b, 1);  // control warp's expect_tx
      sm100::mbar_init(idxe0 + 8 * b, kW);  // every copy warp is done with the block
    }
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), a.tmem_cols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nunits = a.ntiles * a.nco_tiles;
  // unit of this CTA's i-th iteration (nunits past its last one)
  auto unit_at = [&](int i) -> int {
    const int64_t u = (int64_t)blockIdx.x + (int64_t)i * gridDim.x;
    return u < nunits ? (int)u : nunits;
  };

  // tile masks are read ahead so no global-load latency sits at a unit boundary
  auto mask_of = [&](int unit) -> uint32_t { return unit < nunits ? __ldg(a.tile_mask + unit / a.nco_tiles) : 0u; };
  if (warp >= kCopyWarp0 && warp < kControlWarp) {
    // ----------------------------- copy warps -----------------------------
    // All copy warps fill every stage together: warp w owns tile rows
    // [w*RW, (w+1)*RW). Lane (rsub, j) copies 16-byte vector j of rows
    // w*RW + rsub*RPL + p (p < RPL): its RPL source indices are contiguous
    // in the shared index block and each warp instruction moves 32/CPR
    // whole rows. Each lane publishes its copies with
    // cp.async.mbarrier.arrive.noinc, so up to S stages are in flight.
    constexpr int CPR = RB / 16;          // 16-byte vectors per row
    constexpr int RW = kTileRows / kW;    // rows per warp
    constexpr int RPL = RW * CPR / 32;    // rows per lane
    constexpr int EPV = 16 / ES;          // elements per vector
    const int cw = warp - kCopyWarp0;
    const int j = lane % CPR, rsub = lane / CPR;
    const int row0 = cw * RW + rsub * RPL;
    uint32_t soff[RPL];
#pragma unroll
    for (int p = 0; p < RPL; p++) soff[p] = swizzle_off((row0 + p) * RB + j * 16, RB);
    const uint32_t row_stride = (uint32_t)(a.ci * ES);
    const int64_t lo_delta = kSplit ? (a.x_lo - a.x) : 0;
    const int G = a.group;
    uint32_t s = 0, ph = 0, t = 0, cit = 0;
    bool ok = true;
    uint32_t km_next = mask_of(unit_at(0));
    for (int i = 0, u = unit_at(0); u < nunits && ok; u = unit_at(++i), t++) {
      uint32_t km = km_next;
      km_next = mask_of(unit_at(i + 1));
      const int npairs = __popc(km) * a.nchunks;
      if (npairs > 0 && !warp_wait(idxf0 + 8 * (t & 1), (t >> 1) & 1, abort, a.err)) {
        ok = false;
        break;
      }
      const int32_t *idx_t = idx_buf + (t & 1) * kMaxK * kTileRows + row0;
      int c = a.nchunks, slot = -1;
      const uint8_t *gp[RPL];
      uint32_t gs[RPL];
      for (int q = 0; q < npairs && ok;) {
        if (tid == 32 * kCopyWarp0) T2SC_TRACE(0, cit);
        if (!warp_wait(empty0 + 8 * s, ph ^ 1, abort, a.err)) {
          ok = false;
          break;
        }
        if (tid == 32 * kCopyWarp0) T2SC_TRACE(1, cit);
        const uint32_t abase = sbase + s * a.stage_bytes, bar = full0 + 8 * s;
        const int valid = npairs - q < G ? npairs - q : G;
        for (int g = 0; g < valid; g++, q++) {
          if (++c >= a.nchunks) {  // next active offset: its source rows
            c = 0;
            slot++;
            const int32_t *ip = idx_t + slot * kTileRows;
            int32_t src[RPL];
            if (RPL >= 4) {
#pragma unroll
              for (int v = 0; v < RPL / 4; v++) {
                const int4 q4 = reinterpret_cast<const int4 *>(ip)[v];
                src[4 * v] = q4.x, src[4 * v + 1] = q4.y, src[4 * v + 2] = q4.z, src[4 * v + 3] = q4.w;
              }
            } else if (RPL == 2) {
              const int2 q2 = *reinterpret_cast<const int2 *>(ip);
              src[0] = q2.x, src[RPL - 1] = q2.y;
            } else {
              src[0] = ip[0];
            }
#pragma unroll
            for (int p = 0; p < RPL; p++) {
              gp[p] = a.x + (size_t)(src[p] >= 0 ? src[p] : 0) * row_stride + j * 16;
              gs[p] = src[p] >= 0 ? 16u : 0u;
            }
          }
          if (tid == 32 * kCopyWarp0) T2SC_TRACE(10, cit);
          const uint32_t sub = abase + g * a.sub_bytes;
          const bool cvalid = c * BKE + j * EPV < a.ci;
#pragma unroll
          for (int p = 0; p < RPL; p++) {
            const uint32_t sz = cvalid ? gs[p] : 0u;
            if (T2SC_SKIP(1)) {
            } else {
              sm100::cp_async_16(sub + soff[p], gp[p] + c * RB, sz);
              if (kSplit) sm100::cp_async_16(sub + a_tile + soff[p], gp[p] + lo_delta + c * RB, sz);
            }
          }
        }
        if (tid == 32 * kCopyWarp0) T2SC_TRACE(11, cit);
        // arrives on the stage barrier once this lane's copies have landed
        sm100::cp_async_arrive_noinc(bar);
        if (tid == 32 * kCopyWarp0) T2SC_TRACE(6, cit);
        cit++;
        if (++s == (uint32_t)S) {
          s = 0;
          ph ^= 1;
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(idxe0 + 8 * (t & 1));
    }
    sm100::cp_async_wait<0>();
  } else if (warp == kControlWarp) {
    // ---------------------------- control warp ----------------------------
    // Per unit: prefetch the next unit's neighbour-index block (lane i
    // copies the block of the i-th active offset), then issue the weight
    // block of every stage iteration of this unit.
    auto load_idx = [&](int unit, int buf, uint32_t m) {
      const int tl = unit / a.nco_tiles;
      const uint32_t bar = idxf0 + 8 * buf;
      const int nk = __popc(m);
      if (lane == 0) sm100::mbar_arrive_expect_tx(bar, (uint32_t)nk * kTileRows * 4);
      __syncwarp();
      if (lane < nk) {
        const int k = __fns(m, 0, lane + 1);
        const uint32_t dst = sm100::smem_u32(idx_buf + buf * kMaxK * kTileRows) + lane * kTileRows * 4;
        sm100::bulk_g2s(dst, a.nbr_sorted + (int64_t)k * a.n_pad + (int64_t)tl * kTileRows, kTileRows * 4, bar);
      }
    };
    uint32_t it = 0, s = 0, ph = 0, t = 0, n_idx = 0;
    bool ok = true;
    uint32_t km_cur = mask_of(unit_at(0)), km_n1 = mask_of(unit_at(1));
    if (unit_at(0) < nunits) {
      load_idx(unit_at(0), 0, km_cur);  // buffer 0 starts free
      n_idx = 1;
    }
    for (int i = 0, u = unit_at(0); u < nunits && ok; u = unit_at(++i), t++) {
      const int cot = u % a.nco_tiles;
      const uint32_t km = km_cur;
      const uint32_t km_n2 = mask_of(unit_at(i + 2));
      const int u_next = unit_at(i + 1);
      if (u_next < nunits) {
        // the other buffer held unit t-1: wait until every copy warp is done with it
        const uint32_t nb = (t + 1) & 1;
        if (!warp_wait(idxe0 + 8 * nb, (((t + 1) >> 1) & 1) ^ 1, abort, a.err)) {
          ok = false;
          break;
        }
        load_idx(u_next, nb, km_n1);
        n_idx++;
      }
      km_cur = km_n1;
      km_n1 = km_n2;
      // weight blocks: G (k, chunk) pairs per stage, in the copy warps' order
      const int npairs = __popc(km) * a.nchunks;
      uint32_t m = km;
      int c = a.nchunks;
      const uint8_t *wk = a.wimg;
      for (int q = 0; q < npairs && ok;) {
        if (lane == 0) T2SC_TRACE(7, it);
        if (!warp_wait(empty0 + 8 * s, ph ^ 1, abort, a.err)) {
          ok = false;
          break;
        }
        const int valid = npairs - q < a.group ? npairs - q : a.group;
        const uint32_t bar = full0 + 8 * s, abase = sbase + s * a.stage_bytes;
        if (lane == 0) T2SC_TRACE(8, it);
        if (lane == 0) sm100::mbar_arrive_expect_tx(bar, T2SC_SKIP(8) ? 0u : (uint32_t)valid * a.b_bytes);
        for (int g = 0; g < valid; g++, q++) {
          if (++c >= a.nchunks) {
            c = 0;
            const int k = __ffs(m) - 1;
            m &= m - 1;
            wk = a.wimg + (size_t)((size_t)cot * a.kvol + k) * a.nchunks * a.b_bytes;
          }
          if (lane == 0 && !T2SC_SKIP(8))
            sm100::bulk_g2s(abase + g * a.sub_bytes + a.a_bytes, wk + (size_t)c * a.b_bytes, a.b_bytes, bar);
        }
        it++;
        if (++s == (uint32_t)S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    if (lane == 0) {
      // copies requested but never consumed (abort path) land before exit
      for (uint32_t i2 = t; i2 < n_idx; i2++)
        sm100::mbar_wait_cycles(idxf0 + 8 * (i2 & 1), (i2 >> 1) & 1, kWaitLimit / 8);
      if (!ok) {
        const uint32_t first = it > (uint32_t)S ? it - S : 0;
        for (uint32_t i2 = first; i2 < it; i2++)
          sm100::mbar_wait_cycles(full0 + 8 * (i2 % S), (i2 / S) & 1, kWaitLimit / 8);
      }
    }
  } else if (warp < 4) {
    // ------------------------------ epilogue ------------------------------
    const int q = warp;  // TMEM lane quadrant of this warp
    const int row = 32 * q + lane;
    uint32_t acc_it = 0;
    float part[kSplit ? kTf32MaxBn : 1];
    // the next unit's mask and output row are read one unit ahead
    auto orow_of = [&](int unit) -> int {
      return unit < nunits ? __ldg(a.perm + (int64_t)(unit / a.nco_tiles) * kTileRows + row) : -1;
    };
    uint32_t km_next = mask_of(unit_at(0));
    int orow_next = orow_of(unit_at(0));
    for (int i = 0, u = unit_at(0); u < nunits; u = unit_at(++i)) {
      const int cot = u % a.nco_tiles;
      const uint32_t km = km_next;
      const int orow = orow_next;
      km_next = mask_of(unit_at(i + 1));
      orow_next = orow_of(unit_at(i + 1));
      const int col0 = cot * a.bn;
      if (km == 0) {
        // no offset of the tile has a source (not reachable for submanifold
        // maps, whose centre offset always hits): the epilogue of a zero sum,
        // bias -> SiLU -> residual, still applies
        if (orow >= 0) {
          float z[16];
#pragma unroll
          for (int i = 0; i < 16; i++) z[i] = 0.f;
          for (int cc = 0; cc < a.bn; cc += 16) store16<DT>(a, orow, col0 + cc, z);
        }
        continue;
      }
      if (kSplit) {
        // one accumulator drain per kernel offset, summed in f32 registers
#pragma unroll
        for (int i = 0; i < kTf32MaxBn; i++) part[i] = 0.f;
        bool ok = true;
        for (int kk = __popc(km); kk > 0; kk--) {
          const uint32_t b = acc_it & 1;
          if (!warp_wait(tfull0 + 8 * b, (acc_it >> 1) & 1, abort, a.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + b * a.bn;
#pragma unroll
          for (int cc = 0; cc < kTf32MaxBn; cc += 16) {
            if (cc < a.bn) {
              uint32_t r[16];
              sm100::tmem_ld16(tbase + cc, r);
              sm100::tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; i++) part[cc + i] += __uint_as_float(r[i]);
            }
          }
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(tempty0 + 8 * b);
          acc_it++;
        }
        if (!ok) break;
        if (orow >= 0 && !T2SC_SKIP(4)) {
#pragma unroll
          for (int cc = 0; cc < kTf32MaxBn; cc += 16) {
            if (cc < a.bn) {
              float v[16];
#pragma unroll
              for (int i = 0; i < 16; i++) v[i] = part[cc + i];
              store16<DT>(a, orow, col0 + cc, v);
            }
          }
        }
        continue;
      }
      const uint32_t b = acc_it & 1;
      if (tid == 0) T2SC_TRACE(4, acc_it);
      if (!warp_wait(tfull0 + 8 * b, (acc_it >> 1) & 1, abort, a.err)) break;
      if (tid == 0) T2SC_TRACE(5, acc_it);
      sm100::tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + b * a.bn;
      for (int cc = 0; cc < a.bn; cc += 16) {
        uint32_t r[16];
        sm100::tmem_ld16(tbase + cc, r);
        sm100::tmem_ld_wait();
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; i++) acc[i] = __uint_as_float(r[i]);
        if (orow >= 0 && !T2SC_SKIP(4)) store16<DT>(a, orow, col0 + cc, acc);
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(tempty0 + 8 * b);
      acc_it++;
    }
  } else {
    // ----------------------------- MMA issuer -----------------------------
    // The whole warp runs this loop with warp-uniform values (waits agreed
    // by vote); elect.sync picks the lane that issues each tcgen05 op.
    {
      const uint32_t idesc =
          sm100::instr_desc(kSplit ? 2u : (DT == T2SC_DT_BF16 ? 1u : 0u), (uint32_t)a.bn);
      // descriptors of stage 0; a stage or k-step offset is added to the
      // 14-bit start-address field (all of shared memory fits in it)
      const uint64_t dA = sm100::smem_desc(sbase, RB), dB = sm100::smem_desc(sbase + a.a_bytes, RB);
      uint32_t s = 0, ph = 0, acc_it = 0, mit = 0;
      bool ok = true;
      uint32_t km_next = mask_of(unit_at(0));
      for (int i = 0, u = unit_at(0); u < nunits && ok; u = unit_at(++i)) {
        const uint32_t km = km_next;
        km_next = mask_of(unit_at(i + 1));
        if (km == 0) continue;
        const int nk = __popc(km);
        // split-TF32: one accumulator (and one drain) per offset (G = 1);
        // otherwise one per unit. A stage holds up to G (k, chunk) pairs.
        const int groups = kSplit ? nk : 1, pairs_per_group = kSplit ? a.nchunks : nk * a.nchunks;
        for (int gi = 0; gi < groups && ok; gi++) {
          const uint32_t b = acc_it & 1;
          if (!warp_wait(tempty0 + 8 * b, ((acc_it >> 1) & 1) ^ 1, abort, a.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t dtm = tmem + b * a.bn;
          uint32_t accum = 0;
          for (int q = 0; q < pairs_per_group; q += a.group) {
            if (lane == 0) T2SC_TRACE(2, mit);
            if (!warp_wait(full0 + 8 * s, ph, abort, a.err)) {
              ok = false;
              break;
            }
            if (lane == 0) T2SC_TRACE(9, mit);
            sm100::tc_fence_after();
            if (lane == 0) T2SC_TRACE(12, mit);
            const int valid = pairs_per_group - q < a.group ? pairs_per_group - q : a.group;
            for (int g = 0; g < valid; g++) {
              const uint64_t so = (s * a.stage_bytes + g * a.sub_bytes) >> 4;
#pragma unroll
              for (int kk = 0; kk < RB / 32; kk++) {
                const uint64_t ahi = dA + so + kk * 2, bhi = dB + so + kk * 2;
                if (T2SC_SKIP(2)) {
                } else if (kSplit) {
                  const uint64_t alo = ahi + (a_tile >> 4), blo = bhi + (b_tile >> 4);
                  sm100::mma_tf32_elect(dtm, alo, bhi, idesc, accum);
                  sm100::mma_tf32_elect(dtm, ahi, blo, idesc, 1u);
                  sm100::mma_tf32_elect(dtm, ahi, bhi, idesc, 1u);
                } else {
                  sm100::mma_f16_elect(dtm, ahi, bhi, idesc, accum);
                }
                accum = 1;
              }
            }
            if (lane == 0) T2SC_TRACE(13, mit);
            sm100::mma_commit_elect(empty0 + 8 * s);
            if (lane == 0) T2SC_TRACE(3, mit);
            mit++;
            if (++s == (uint32_t)S) {
              s = 0;
              ph ^= 1;
            }
          }
          if (!ok) break;
          sm100::mma_commit_elect(tfull0 + 8 * b);
          acc_it++;
        }
      }
      // all issued MMAs retire before TMEM is released
      sm100::mma_commit_elect(mma_done);
      if (lane == 0) sm100::mbar_wait_cycles(mma_done, 0, kWaitLimit / 8);
    }
    __syncwarp();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, a.tmem_cols);
  }
}

// x = hi + lo with hi the nearest TF32 value (cvt.rna) and lo exact in f32.
__global__ void split_tf32_kernel(const float4 *__restrict__ x, float4 *__restrict__ hi, float4 *__restrict__ lo,
                                  int64_t n4) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 v = x[i], h, l;
  float *pv = &v.x, *ph = &h.x, *pl = &l.x;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t t;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(pv[q]));
    ph[q] = __uint_as_float(t);
    pl[q] = pv[q] - ph[q];
  }
  hi[i] = h;
  lo[i] = l;
}

template <int DT, int RB>
int launch_tc(t2sc_conv *cv, const TcArgs &args, int grid, size_t smem, std::string &err) {
  auto kfn = conv_tc_kernel<DT, RB>;
  // set the shared-memory opt-in once per instantiation and size (a host-only
  // call kept out of the per-launch path, e.g. during stream capture)
  static int attr_smem[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || attr_smem[dev] < (int)smem) {
    T2SC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "tc smem attr");
    if (dev >= 0 && dev < 64) attr_smem[dev] = (int)smem;
  }
#if T2SC_CONV_DIAGNOSTICS
  const char *trace_path = getenv("T2SC_CONV_TRACE");
  if (trace_path) {  // diagnostics only: allocates, synchronises and writes a file
    TcArgs t = args;
    const size_t bytes = 14 * kTraceN * sizeof(long long);
    T2SC_CUDA(cudaMalloc((void **)&t.trace, bytes), "trace");
    T2SC_CUDA(cudaMemset(t.trace, 0, bytes), "trace");
    kfn<<<grid, Roles<DT, RB>::kThreads, smem, cv->ctx->stream>>>(t);
    T2SC_LAUNCHED(cv->ctx, "conv_tc");
    std::vector<long long> h(14 * kTraceN);
    T2SC_CUDA(cudaMemcpyAsync(h.data(), t.trace, bytes, cudaMemcpyDeviceToHost, cv->ctx->stream), "trace");
    T2SC_CUDA(cudaStreamSynchronize(cv->ctx->stream), "trace");
    cudaFree(t.trace);
    if (FILE *f = fopen(trace_path, "wb")) {
      fwrite(h.data(), 1, bytes, f);
      fclose(f);
    }
    return T2SC_OK;
  }
#endif
  kfn<<<grid, Roles<DT, RB>::kThreads, smem, cv->ctx->stream>>>(args);
  T2SC_LAUNCHED(cv->ctx, "conv_tc");
  return T2SC_OK;
}

}  // namespace

// TF32 value nearest to f (ties away from zero), as cvt.rna.tf32.f32 rounds.
static float tf32_round_host(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & ~0x1fffu;
  memcpy(&f, &u, 4);
  return f;
}

// Chooses the tile shape and builds the pre-swizzled weight image: one
// block per (co tile, k, ci chunk) holding bn rows (output channels) x
// row_bytes (a chunk of input channels), exactly the B stage's smem image.
// In the split-TF32 mode each block is the hi image followed by the lo image.
int conv_tc_prepare(t2sc_conv *cv, const float *w, std::string &err) {
  const int co = cv->co, ci = cv->ci, K = cv->kvol;
  const bool f32 = cv->dtype == T2SC_DT_F32;
  const int es = f32 ? 4 : 2, na = f32 ? 2 : 1;
  const int ci_bytes = ci * es;
  // 16-bit modes stream 128-byte rows; the split-TF32 mode keeps two A and
  // two B tiles per stage, so it uses 64-byte rows to fit four stages
  const int max_rb = f32 ? 64 : 128;
  cv->row_bytes = ci_bytes >= max_rb ? max_rb : (ci_bytes > 32 ? 64 : 32);
  const int bke = cv->row_bytes / es;
  cv->nchunks = (ci + bke - 1) / bke;
  const int bn_max = f32 ? 128 : 256;
  int bn = 0;
  for (int d = bn_max; d >= 16; d -= 16)
    if (co % d == 0) {
      bn = d;
      break;
    }
  cv->bn = bn;
  cv->nco_tiles = co / bn;
  const size_t tile = (size_t)bn * cv->row_bytes, bbytes = tile * na;
  const size_t total = bbytes * cv->nco_tiles * K * cv->nchunks;
  std::vector<uint8_t> img(total, 0);
  for (int nt = 0; nt < cv->nco_tiles; nt++)
    for (int k = 0; k < K; k++)
      for (int c = 0; c < cv->nchunks; c++) {
        uint8_t *blk = img.data() + ((size_t)(nt * K + k) * cv->nchunks + c) * bbytes;
        for (int r = 0; r < bn; r++)
          for (int e = 0; e < bke; e++) {
            const int o = nt * bn + r, i = c * bke + e;
            const float v = (i < ci) ? w[((size_t)o * K + k) * ci + i] : 0.0f;
            const uint32_t off = swizzle_off((uint32_t)(r * cv->row_bytes + e * es), cv->row_bytes);
            if (f32) {
              const float hi = tf32_round_host(v), lo = v - hi;
              memcpy(blk + off, &hi, 4);
              memcpy(blk + tile + off, &lo, 4);
            } else if (cv->dtype == T2SC_DT_BF16) {
              __nv_bfloat16 h = __float2bfloat16_rn(v);
              memcpy(blk + off, &h, 2);
            } else {
              __half h = __float2half_rn(v);
              memcpy(blk + off, &h, 2);
            }
          }
      }
  T2SC_CUDA(cudaMalloc(&cv->d_wtc, total), "conv weights");
  T2SC_CUDA(cudaMemcpy(cv->d_wtc, img.data(), total, cudaMemcpyHostToDevice), "conv weights upload");
  return T2SC_OK;
}

int conv_tc_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags, const void *residual,
                   std::string &err) {
  if (m->n == 0) return T2SC_OK;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(residual)) & 15) {
    err = "feature buffers must be 16-byte aligned";
    return T2SC_ERR_INVALID;
  }
  TcArgs a;
  a.x = static_cast<const uint8_t *>(x);
  a.x_lo = nullptr;
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
#if T2SC_CONV_DIAGNOSTICS
  static const int debug_bits = [] {
    const char *e = getenv("T2SC_CONV_DEBUG");
    return e ? atoi(e) : 0;
  }();
  a.debug = debug_bits;
  a.trace = nullptr;
#endif
  int cols = 32;
  while (cols < 2 * cv->bn) cols <<= 1;
  a.tmem_cols = cols;
  const int na = cv->dtype == T2SC_DT_F32 ? 2 : 1;
  a.a_bytes = kTileRows * cv->row_bytes * na;
  a.b_bytes = (uint32_t)cv->bn * cv->row_bytes * na;
  a.sub_bytes = (a.a_bytes + a.b_bytes + 1023u) & ~1023u;
  const int idx_bytes = 2 * kMaxK * kTileRows * 4;  // double-buffered tile index blocks
  // CTAs per SM: 2 independent pipelines when both fit (TMEM <= 256 columns
  // each, half the shared memory each), else 1.
  static const int ctas_env = [] {
    const char *e = getenv("T2SC_CONV_CTAS");
    return e ? atoi(e) : kDefaultCtasPerSm;
  }();
  int ctas = (ctas_env >= 2 && cols <= 256 && cv->dtype != T2SC_DT_F32) ? 2 : 1;
  // two CTAs only when half the shared memory still holds kMinStages stages
  if (ctas == 2 && (int)(kSmemHalf - idx_bytes - 1280) / (int)a.sub_bytes < kMinStages) ctas = 1;
  const int avail = (ctas == 2 ? kSmemHalf : kSmemMax) - idx_bytes - 1280;
  // Small pairs are grouped so that one stage carries up to ~48 KB: the
  // per-stage handshake is then paid once per several MMA k-steps.
  // Split-TF32 drains per offset, so it keeps one pair per stage.
  int G = 1;
  if (cv->dtype != T2SC_DT_F32)
    while (G < 4 && (int)((G + 1) * a.sub_bytes) <= 48 * 1024 && avail / (int)((G + 1) * a.sub_bytes) >= 4) G++;
  a.group = G;
  a.stage_bytes = G * a.sub_bytes;
  int S = avail / (int)a.stage_bytes;
  if (S > 8) S = 8;
  if (S < kMinStages) {
    err = "conv tile does not fit shared memory";
    return T2SC_ERR_UNSUPPORTED;
  }
  a.stages = S;
  // stages + index blocks + barriers/slots + alignment slack; with one CTA
  // per SM never below 120 KB, so that it alone owns the SM (and its TMEM).
  size_t smem = (size_t)S * a.stage_bytes + idx_bytes + 256 + 1024;
  if (ctas == 1 && smem < 120 * 1024) smem = 120 * 1024;
  const int64_t nunits = (int64_t)a.ntiles * a.nco_tiles;
  const int64_t slots = (int64_t)cv->ctx->num_sms * ctas;
  const int grid = (int)(nunits < slots ? nunits : slots);
  if (cv->dtype == T2SC_DT_F32) {
    // split x into TF32 hi/lo parts in the context's grow-only scratch
    // (stream-ordered: calls on the context's stream reuse it in turn; it
    // is reallocated only when a larger input arrives)
    t2sc_ctx *ctx = cv->ctx;
    cudaStream_t st = ctx->stream;
    const int64_t cnt = m->n_src * (int64_t)cv->ci;
    const size_t need = (size_t)cnt * 8;
    if (ctx->stage_cap[0] < need) {
      if (ctx->stage[0]) cudaFreeAsync(ctx->stage[0], st);
      ctx->stage[0] = nullptr;
      ctx->stage_cap[0] = 0;
      T2SC_CUDA(cudaMallocAsync(&ctx->stage[0], need, st), "split scratch");
      ctx->stage_cap[0] = need;
    }
    float *split = static_cast<float *>(ctx->stage[0]);
    const int64_t n4 = cnt / 4;
    split_tf32_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>((const float4 *)x, (float4 *)split,
                                                                     (float4 *)(split + cnt), n4);
    T2SC_LAUNCHED(cv->ctx, "split_tf32");
    a.x = reinterpret_cast<const uint8_t *>(split);
    a.x_lo = reinterpret_cast<const uint8_t *>(split + cnt);
    int rc = cv->row_bytes == 64 ? launch_tc<kModeTf32x3, 64>(cv, a, grid, smem, err)
                                 : launch_tc<kModeTf32x3, 32>(cv, a, grid, smem, err);
    return rc;
  }
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
