// Staged-window SubM conv on the sm_100a tensor cores, for 16-bit features
// with Ci = Co = 64 (the 512^3 decoder level).
//
// The other conv kernel (conv_tc.cu) gathers every (tile, offset) operand
// row from L2 with 16-byte cp.async copies; at C = 64 those copies cap the
// kernel (the gather path moves ~23 bytes per clock per SM). Here a tile is
// 128 consecutive target rows in their own (coordinate) order, whose
// distinct source rows are few (about 3.5 per target at the 512^3 shell)
// and sit in about ten runs of consecutive rows. Per tile:
//
//   loader warp   bulk-copies the tile's source runs into a shared-memory
//                 window (one copy per run, double-buffered across tiles)
//                 and streams the weight block of every active offset;
//   builder warps (4, one per TMEM lane quadrant) build each (tile, offset)
//                 A operand in tensor memory: thread m reads its source row
//                 from the window (eight 16-byte loads, each lane starting at
//                 its own chunk so a quarter warp touches 8 distinct banks)
//                 and stores the 64 values to TMEM lane m with tcgen05.st;
//                 rows without a source store zeros;
//   MMA warp      one lane issues tcgen05.mma with A from TMEM and B from
//                 shared memory into a double-buffered TMEM accumulator;
//   epilogue (4)  tcgen05.ld, bias, SiLU, residual, convert, store.
//
// TMEM: accumulators 2 x 64 columns, A stages 8 x 32 columns (512 in all:
// one CTA per SM). Shared memory: 2 windows x 512 rows x 128 B + 8 weight
// stages x 8 KB. Every mbarrier wait is bounded; on a timeout the CTA sets
// the error flag, lets its copies land, frees TMEM and returns.
#include <stdio.h>
#include <stdlib.h>

#include <vector>

#include "epilogue.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace t2sc {
namespace {

// Warp roles for NB builder sets: warps [0, 4NB) build A operands (warp w
// serves TMEM lane quadrant w % 4; set w / 4 takes every NB-th operand),
// then 4 epilogue warps, the loader warp and the MMA warp.
template <int NB>
struct WRoles {
  static constexpr int kEpi0 = 4 * NB, kLoader = 4 * NB + 4, kMma = 4 * NB + 5, kThreads = 32 * (4 * NB + 6);
};
// G kernel offsets per pipeline stage: an A stage is G x 32 TMEM columns,
// a B stage G weight blocks. Stages per ring for G = 1, 2, 3.
// kNacc independent accumulators per tile: consecutive MMA k-steps write
// different ones (an MMA into the accumulator the previous MMA writes
// waits for it), and the epilogue adds them.
constexpr int kNacc = 2;
constexpr int kACol = 2 * kNacc * 64;  // TMEM columns: accumulators [2 buffers][kNacc][64], then A stages
template <int G>
struct WStages {
  static constexpr int kS0 = (512 - kACol) / (32 * G);
  static constexpr int kS = kS0 > 8 ? 8 : kS0;               // A stages (TMEM)
  static constexpr int kSB = G == 1 ? 8 : (G == 2 ? 5 : 3);  // B stages (shared memory)
};
constexpr uint32_t kSlotBytes = 7168;  // a tile's slot block: K (<= 27) x 128 int16, rounded up
constexpr int kRowB = 128;       // bytes per feature row (64 x 16-bit)
constexpr uint32_t kBBytes = 64 * kRowB;       // one weight block (64 output channels x 64 inputs)
constexpr uint32_t kWinBytes = kWinRows * kRowB;
constexpr long long kWLimit = 4000000000LL;    // ~2 s of SM clocks
constexpr int kAccCol = 0;

struct WinArgs {
  const uint8_t *x;    // [n_src, 64] 16-bit
  uint8_t *y;          // [n, 64]
  const uint8_t *res;  // [n, 64] or null
  const uint8_t *wimg; // weight blocks [k] x 8 KB (pre-swizzled B images)
  const float *bias;   // [64]
  const int16_t *slot16;
  const int32_t *runs, *meta;
  const uint32_t *tmask;
  int64_t n, n_pad;
  int ntiles, co, flags, kvol;
  int wait_mode;  // how a waiting thread polls (sm100::mbar_wait_bounded)
  int *err;
#if T2SC_CONV_DIAGNOSTICS
  int debug;  // 1 skips the window copies, 2 the MMAs, 4 the weight copies, 8 the TMEM stores
  long long *trace;  // per-stage clocks of CTA 0 (T2SC_CONV_TRACE), or null
#endif
};
#ifndef T2SC_CONV_DIAGNOSTICS
#define T2SC_CONV_DIAGNOSTICS 0
#endif
#if T2SC_CONV_DIAGNOSTICS
#define WSKIP(bit) (a.debug & (bit))
constexpr int kWTraceN = 4096;
#define WTRACE(slot, idx)                                                                          \
  do {                                                                                             \
    if (a.trace && blockIdx.x == 0 && (idx) < kWTraceN) a.trace[(slot) * kWTraceN + (idx)] = clock64(); \
  } while (0)
#else
#define WSKIP(bit) false
#define WTRACE(slot, idx) \
  do {                    \
  } while (0)
#endif

__device__ __forceinline__ bool wwait(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int mode) {
  bool ok = sm100::mbar_test_wait(bar, parity);
  if (__all_sync(0xffffffffu, ok)) return true;
  if (!ok) ok = sm100::mbar_wait_bounded(bar, parity, abort, err, kDevErrTimeout, kWLimit, mode);
  return __all_sync(0xffffffffu, ok);
}

// Rotates eight 16-byte chunks right by r (0..7): out[c] = in[(c - r) & 7].
__device__ __forceinline__ void rotate_chunks(uint32_t (&v)[32], int r) {
#pragma unroll
  for (int b = 1; b < 8; b <<= 1) {
    const bool on = r & b;
    uint32_t t[32];
#pragma unroll
    for (int c = 0; c < 8; c++)
#pragma unroll
      for (int w = 0; w < 4; w++) t[4 * c + w] = on ? v[4 * ((c - b) & 7) + w] : v[4 * c + w];
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = t[i];
  }
}

template <int DT, int NB, int G>
__global__ void __launch_bounds__(WRoles<NB>::kThreads, 1) conv_win_kernel(const WinArgs a) {
  constexpr int kWLoader = WRoles<NB>::kLoader, kWMma = WRoles<NB>::kMma, kEpi0 = WRoles<NB>::kEpi0;
  constexpr int kSA = WStages<G>::kS, kSB = WStages<G>::kSB;
  constexpr uint32_t kStageB = G * kBBytes;  // bytes of one B stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *win = smem;                          // [2][kWinBytes]
  const int16_t *sslot = reinterpret_cast<const int16_t *>(smem + 2 * kWinBytes);  // [2][K][128]
  uint8_t *bst = smem + 2 * kWinBytes + 2 * kSlotBytes;  // [kSB][G][kBBytes]
  uint64_t *bars = reinterpret_cast<uint64_t *>(bst + kSB * kStageB);
  // bars: win_full[2], win_empty[2], a_full[kSA], a_empty[kSA], b_full[kSB], b_empty[kSB],
  //       acc_full[2], acc_empty[2], done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 8 + 2 * kSA + 2 * kSB + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const uint32_t wf0 = sm100::smem_u32(bars), we0 = wf0 + 16, af0 = we0 + 16, ae0 = af0 + 8 * kSA,
                 bf0 = ae0 + 8 * kSA, be0 = bf0 + 8 * kSB, cf0 = be0 + 8 * kSB, ce0 = cf0 + 16, done = ce0 + 16;
  const uint32_t win_s = sm100::smem_u32(win), bst_s = sm100::smem_u32(bst), slot_s = win_s + 2 * kWinBytes;
  const uint32_t slot_bytes = (uint32_t)a.kvol * kTileRows * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int b = 0; b < 2; b++) {
      sm100::mbar_init(wf0 + 8 * b, 1);
      sm100::mbar_init(we0 + 8 * b, 4 * NB);  // every builder warp releases the window
      sm100::mbar_init(cf0 + 8 * b, 1);
      sm100::mbar_init(ce0 + 8 * b, 4);
    }
    for (int s = 0; s < kSA; s++) sm100::mbar_init(af0 + 8 * s, 4), sm100::mbar_init(ae0 + 8 * s, 1);
    for (int s = 0; s < kSB; s++) sm100::mbar_init(bf0 + 8 * s, 1), sm100::mbar_init(be0 + 8 * s, 1);
    sm100::mbar_init(done, 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == kWMma) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto mask_of = [&](int t) -> uint32_t { return t < a.ntiles ? __ldg(a.tmask + t) : 0u; };

  if (warp == kWLoader) {
    // ------------------------------ loader ------------------------------
    uint32_t sb = 0, bph = 0, nb = 0;
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x, i++) {
      const int wb = i & 1;
      if (!wwait(we0 + 8 * wb, ((i >> 1) & 1) ^ 1, abort, a.err, a.wait_mode)) {
        ok = false;
        break;
      }
      const int nruns = __ldg(a.meta + 2 * t), rows = __ldg(a.meta + 2 * t + 1);
      // the window rows and the tile's slot block complete the same barrier
      if (lane == 0) WTRACE(8, i);
      if (lane == 0) {
        sm100::mbar_arrive_expect_tx(wf0 + 8 * wb, (WSKIP(1) ? 0u : (uint32_t)rows * kRowB) + slot_bytes);
        sm100::bulk_g2s(slot_s + wb * kSlotBytes, a.slot16 + (int64_t)t * a.kvol * kTileRows, slot_bytes,
                        wf0 + 8 * wb);
      }
      __syncwarp();
      const int32_t *rp = a.runs + (int64_t)t * kWinRunCap * 2;
      for (int r = lane; r < nruns && !WSKIP(1); r += 32) {
        const int src0 = __ldg(rp + 2 * r), slot0 = __ldg(rp + 2 * r + 1);
        const int next = r + 1 < nruns ? __ldg(rp + 2 * r + 3) : rows;
        sm100::bulk_g2s(win_s + wb * kWinBytes + slot0 * kRowB, a.x + (int64_t)src0 * kRowB,
                        (uint32_t)(next - slot0) * kRowB, wf0 + 8 * wb);
      }
      // weight blocks of the tile's offsets, G per stage, in the builders' order
      for (uint32_t m = mask_of(t); m && ok;) {
        const int valid = __popc(m) < G ? __popc(m) : G;
        const int k = lane < valid ? __fns(m, 0, lane + 1) : 0;  // the lane-th active offset
        for (int g = 0; g < valid; g++) m &= m - 1;
        if (!wwait(be0 + 8 * sb, bph ^ 1, abort, a.err, a.wait_mode)) {
          ok = false;
          break;
        }
        if (lane == 0) WTRACE(7, nb);
        if (lane == 0) sm100::mbar_arrive_expect_tx(bf0 + 8 * sb, WSKIP(4) ? 0u : valid * kBBytes);
        __syncwarp();
        if (lane < valid && !WSKIP(4))
          sm100::bulk_g2s(bst_s + sb * kStageB + lane * kBBytes, a.wimg + (size_t)k * kBBytes, kBBytes, bf0 + 8 * sb);
        nb++;
        if (++sb == kSB) sb = 0, bph ^= 1;
      }
    }
    if (lane == 0 && !ok) {
      // copies requested but maybe never consumed land before exit
      for (int b = 0; b < 2; b++) sm100::mbar_wait_cycles(wf0 + 8 * b, 0, kWLimit / 16);
      for (uint32_t q = nb > (uint32_t)kSB ? nb - kSB : 0; q < nb; q++)
        sm100::mbar_wait_cycles(bf0 + 8 * (q % kSB), (q / kSB) & 1, kWLimit / 16);
    }
  } else if (warp < kEpi0) {
    // ----------------------------- builders -----------------------------
    const int q = warp & 3, set = warp >> 2, row = 32 * q + lane, rot = lane & 7;
    uint32_t pc = 0;  // operands of this CTA so far (all sets)
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x, i++) {
      const int wb = i & 1;
      if (!wwait(wf0 + 8 * wb, (i >> 1) & 1, abort, a.err, a.wait_mode)) {
        ok = false;
        break;
      }
      const uint8_t *wbase = win + wb * kWinBytes;
      for (uint32_t m = mask_of(t); m; pc++) {
        const int valid = __popc(m) < G ? __popc(m) : G;
        uint32_t ks = m;  // this stage's offsets: the next `valid` bits of m
        for (int g = 0; g < valid; g++) m &= m - 1;
        if ((int)(pc % NB) != set) continue;
        const uint32_t sa = pc % kSA, aph = (pc / kSA) & 1;
        if (warp == 0 && lane == 0) WTRACE(0, pc);
        if (!wwait(ae0 + 8 * sa, aph ^ 1, abort, a.err, a.wait_mode)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        for (int g = 0; g < valid; g++, ks &= ks - 1) {
          const int slot = sslot[wb * (kSlotBytes / 2) + (__ffs(ks) - 1) * kTileRows + row];
          uint32_t v[32];
          if (slot >= 0 && !WSKIP(32)) {
            const uint8_t *rowp = wbase + slot * kRowB;
#pragma unroll
            for (int j = 0; j < 8; j++) {  // chunk (j + rot) & 7: the 8 lanes of a quarter warp hit 8 bank groups
              const uint4 c = *reinterpret_cast<const uint4 *>(rowp + (((j + rot) & 7) << 4));
              v[4 * j] = c.x, v[4 * j + 1] = c.y, v[4 * j + 2] = c.z, v[4 * j + 3] = c.w;
            }
            if (!WSKIP(16)) rotate_chunks(v, rot);
          } else {
#pragma unroll
            for (int w = 0; w < 32; w++) v[w] = 0u;
          }
          if (!WSKIP(8)) sm100::tmem_st32(tmem + ((uint32_t)(32 * q) << 16) + kACol + 32 * (G * sa + g), v);
        }
        if (warp == 0 && lane == 0) WTRACE(1, pc);
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(af0 + 8 * sa);
        if (warp == 0 && lane == 0) WTRACE(2, pc);
      }
      if (!ok) break;
      // this warp is done with the window: its reads are ordered before the
      // bulk copies (async proxy) that will refill the buffer
      sm100::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(we0 + 8 * wb);
    }
  } else if (warp < kEpi0 + 4) {
    // ----------------------------- epilogue -----------------------------
    const int q = warp - kEpi0, row = 32 * q + lane;
    uint32_t acc_it = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x) {
      const int64_t p = (int64_t)t * kTileRows + row;
      const int orow = p < a.n ? (int)p : -1;
      if (mask_of(t) == 0) {  // no sources at all: the epilogue of a zero sum
        if (orow >= 0) {
          float z[16];
#pragma unroll
          for (int c = 0; c < 16; c++) z[c] = 0.f;
          for (int cc = 0; cc < 64; cc += 16) store16<DT>(a, orow, cc, z);
        }
        continue;
      }
      const uint32_t b = acc_it & 1;
      if (!wwait(cf0 + 8 * b, (acc_it >> 1) & 1, abort, a.err, a.wait_mode)) break;
      sm100::tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + kAccCol + kNacc * 64 * b;
      const int used = 4 * __popc(mask_of(t)) < kNacc ? 4 * __popc(mask_of(t)) : kNacc;
#pragma unroll
      for (int cc = 0; cc < 64; cc += 16) {
        uint32_t r[16];
        sm100::tmem_ld16(tb + cc, r);
        sm100::tmem_ld_wait();
        float acc[16];
#pragma unroll
        for (int c = 0; c < 16; c++) acc[c] = __uint_as_float(r[c]);
        for (int j = 1; j < used; j++) {
          sm100::tmem_ld16(tb + 64 * j + cc, r);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; c++) acc[c] += __uint_as_float(r[c]);
        }
        if (orow >= 0) store16<DT>(a, orow, cc, acc);
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(ce0 + 8 * b);
      acc_it++;
    }
  } else {
    // -------------------------------- MMA --------------------------------
    if (lane == 0) {
      const uint32_t idesc = sm100::instr_desc(DT == T2SC_DT_BF16 ? 1u : 0u, 64u);
      const uint64_t dB = sm100::smem_desc(bst_s, kRowB);
      uint32_t sa = 0, aph = 0, sb = 0, bph = 0, acc_it = 0, mst = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x) {
        uint32_t m = mask_of(t);
        if (!m) continue;
        const uint32_t b = acc_it & 1;
        if (!sm100::mbar_wait_bounded(ce0 + 8 * b, ((acc_it >> 1) & 1) ^ 1, abort, a.err, kDevErrTimeout, kWLimit, a.wait_mode)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem + kAccCol + kNacc * 64 * b;
        int kstep = 0;
        while (m) {
          const int valid = __popc(m) < G ? __popc(m) : G;
          for (int g = 0; g < valid; g++) m &= m - 1;
          WTRACE(3, mst);
          if (!sm100::mbar_wait_bounded(af0 + 8 * sa, aph, abort, a.err, kDevErrTimeout, kWLimit, a.wait_mode)) {
            ok = false;
            break;
          }
          WTRACE(4, mst);
          if (!sm100::mbar_wait_bounded(bf0 + 8 * sb, bph, abort, a.err, kDevErrTimeout, kWLimit, a.wait_mode)) {
            ok = false;
            break;
          }
          WTRACE(5, mst);
          sm100::tc_fence_after();
          for (int g = 0; g < valid; g++) {
            const uint32_t at = tmem + kACol + 32 * (G * sa + g);
            const uint64_t bd = dB + ((uint64_t)(sb * kStageB + g * kBBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {  // K = 64 in four steps of 16 (8 TMEM columns, 32 bytes of B)
              if (!WSKIP(2))
                sm100::mma_f16_ta(d + 64 * (kstep % kNacc), at + 8 * kk, bd + 2 * kk, idesc, kstep >= kNacc ? 1u : 0u);
              kstep++;
            }
          }
          sm100::mma_commit(ae0 + 8 * sa);
          sm100::mma_commit(be0 + 8 * sb);
          WTRACE(6, mst);
          mst++;
          if (++sa == kSA) sa = 0, aph ^= 1;
          if (++sb == kSB) sb = 0, bph ^= 1;
        }
        if (!ok) break;
        sm100::mma_commit(cf0 + 8 * b);
        acc_it++;
      }
      sm100::mma_commit(done);  // every issued MMA retires before TMEM is released
      sm100::mbar_wait_cycles(done, 0, kWLimit / 8);
    }
    __syncwarp();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == kWMma) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

template <int DT, int NB, int G>
int launch_win(t2sc_conv *cv, const WinArgs &a, int grid, std::string &err) {
  auto kfn = conv_win_kernel<DT, NB, G>;
  const size_t smem = 2 * (size_t)kWinBytes + 2 * (size_t)kSlotBytes + WStages<G>::kSB * (size_t)G * kBBytes + 64 * 8 +
                      1024;
  static int attr_set[64] = {};  // one per instantiation: the shared-memory opt-in, set once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    T2SC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "win smem attr");
    if (dev >= 0 && dev < 64) attr_set[dev] = 1;
  }
#if T2SC_CONV_DIAGNOSTICS
  if (const char *path = getenv("T2SC_CONV_TRACE")) {  // diagnostics only: allocates, synchronises, writes a file
    WinArgs t = a;
    const size_t bytes = 10 * kWTraceN * sizeof(long long);
    T2SC_CUDA(cudaMalloc((void **)&t.trace, bytes), "trace");
    T2SC_CUDA(cudaMemset(t.trace, 0, bytes), "trace");
    kfn<<<grid, WRoles<NB>::kThreads, smem, cv->ctx->stream>>>(t);
    T2SC_LAUNCHED(cv->ctx, "conv_win");
    std::vector<long long> h(10 * kWTraceN);
    T2SC_CUDA(cudaMemcpyAsync(h.data(), t.trace, bytes, cudaMemcpyDeviceToHost, cv->ctx->stream), "trace");
    T2SC_CUDA(cudaStreamSynchronize(cv->ctx->stream), "trace");
    cudaFree(t.trace);
    if (FILE *f = fopen(path, "wb")) {
      fwrite(h.data(), 1, bytes, f);
      fclose(f);
    }
    return T2SC_OK;
  }
#endif
  kfn<<<grid, WRoles<NB>::kThreads, smem, cv->ctx->stream>>>(a);
  T2SC_LAUNCHED(cv->ctx, "conv_win");
  return T2SC_OK;
}

}  // namespace

int conv_win_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags, const void *residual,
                    std::string &err) {
  if (cv->dtype == T2SC_DT_F32 || !cv->tc_path || cv->ci != 64 || cv->co != 64 || cv->row_bytes != kRowB ||
      cv->bn != 64 || cv->nchunks != 1 || m->kvol > 27 || !m->slot16)
    return T2SC_ERR_UNSUPPORTED;
  int ok = 0;
  int rc = map_win_ok(m, &ok, err);
  if (rc != T2SC_OK) return rc;
  if (!ok) return T2SC_ERR_UNSUPPORTED;
  if (m->n == 0) return T2SC_OK;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(residual)) & 15) {
    err = "feature buffers must be 16-byte aligned";
    return T2SC_ERR_INVALID;
  }
  WinArgs a;
  a.x = static_cast<const uint8_t *>(x);
  a.y = static_cast<uint8_t *>(y);
  a.res = static_cast<const uint8_t *>(residual);
  a.wimg = static_cast<const uint8_t *>(cv->d_wtc);
  a.bias = cv->d_bias;
  a.slot16 = m->slot16;
  a.runs = m->win_runs;
  a.meta = m->win_meta;
  a.tmask = m->tile_mask_nat;
  a.n = m->n;
  a.n_pad = m->n_pad;
  a.ntiles = (int)m->ntiles;
  a.co = cv->co;
  a.flags = flags;
  a.kvol = m->kvol;
  static const int wm_env = getenv("T2SC_WAIT_MODE") ? atoi(getenv("T2SC_WAIT_MODE")) : 0;
  a.wait_mode = wm_env;
  a.err = cv->ctx->d_err;
#if T2SC_CONV_DIAGNOSTICS
  a.debug = getenv("T2SC_CONV_DEBUG") ? atoi(getenv("T2SC_CONV_DEBUG")) : 0;
  a.trace = nullptr;
#endif
  const int grid = (int)(m->ntiles < cv->ctx->num_sms ? m->ntiles : cv->ctx->num_sms);
  static const int nb_env = getenv("T2SC_WIN_SETS") ? atoi(getenv("T2SC_WIN_SETS")) : 4;
  static const int g_env = getenv("T2SC_WIN_GROUP") ? atoi(getenv("T2SC_WIN_GROUP")) : 2;
  const bool bf = cv->dtype == T2SC_DT_BF16;
#define T2SC_WIN(NB, G) \
  return bf ? launch_win<T2SC_DT_BF16, NB, G>(cv, a, grid, err) : launch_win<T2SC_DT_F16, NB, G>(cv, a, grid, err)
  if (nb_env == 2) {
    if (g_env == 1) T2SC_WIN(2, 1);
    if (g_env == 3) T2SC_WIN(2, 3);
    T2SC_WIN(2, 2);
  }
  if (g_env == 1) T2SC_WIN(4, 1);
  if (g_env == 3) T2SC_WIN(4, 3);
  T2SC_WIN(4, 2);
#undef T2SC_WIN
}

}  // namespace t2sc
