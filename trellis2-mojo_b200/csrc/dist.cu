// Multi-GPU data plane of the library: the z-slab partition of a voxel set
// (host code) and the per-layer halo exchange over NCCL (one communicator
// per slab group, send/recv grouped on the context's stream), with bounded
// waits that abort a communicator whose peer stopped answering.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy
// the process has already loaded), so the library loads without NCCL and
// never brings a second NCCL build into a process that has one.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"

struct t2sc_comm {
  t2sc_ctx *ctx = nullptr;
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0;
  bool aborted = false;
};

namespace {

struct NcclApi {
  void *handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own NCCL, if any
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    api.handle = h;
#define T2SC_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    T2SC_SYM(GetUniqueId, "ncclGetUniqueId");
    T2SC_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    T2SC_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    T2SC_SYM(CommAbort, "ncclCommAbort");
    T2SC_SYM(CommFinalize, "ncclCommFinalize");
    T2SC_SYM(CommDestroy, "ncclCommDestroy");
    T2SC_SYM(GroupStart, "ncclGroupStart");
    T2SC_SYM(GroupEnd, "ncclGroupEnd");
    T2SC_SYM(Send, "ncclSend");
    T2SC_SYM(Recv, "ncclRecv");
    T2SC_SYM(GetErrorString, "ncclGetErrorString");
#undef T2SC_SYM
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort &&
             api.CommFinalize && api.CommDestroy && api.GroupStart && api.GroupEnd && api.Send && api.Recv &&
             api.GetErrorString;
  });
  return api;
}

int fail(t2sc_ctx *ctx, int code, const std::string &msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

std::string nccl_msg(const char *what, ncclResult_t r) {
  return std::string(what) + ": " + (nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error");
}

// Polls a non-blocking communicator until its pending operation finished,
// it reported an error, or timeout_ms passed (then the communicator is
// aborted). Returns T2SC_OK, T2SC_ERR_CUDA or T2SC_ERR_TIMEOUT.
int wait_comm_ready(t2sc_comm *c, int timeout_ms, std::string &err) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return T2SC_OK;
    if (st != ncclInProgress) {
      err = nccl_msg("NCCL", st);
      return T2SC_ERR_CUDA;
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      err = "NCCL operation did not finish within the timeout; communicator aborted";
      return T2SC_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

extern "C" {

int t2sc_partition_zslab(const int32_t *coords, int64_t n, int world, int rank, int depth, int64_t *rows,
                         int64_t cap, int64_t *counts) {
  if (!counts || n < 0 || world < 1 || rank < 0 || rank >= world || depth < 1 || (n > 0 && !coords))
    return T2SC_ERR_INVALID;
  for (int i = 0; i < 6; i++) counts[i] = 0;
  if (n == 0) return T2SC_OK;
  int64_t zmin = coords[3], zmax = coords[3];
  for (int64_t r = 1; r < n; r++) {
    zmin = std::min<int64_t>(zmin, coords[4 * r + 3]);
    zmax = std::max<int64_t>(zmax, coords[4 * r + 3]);
  }
  zmax += 1;
  int64_t lo = zmin, hi = zmax;
  if (world > 1) {
    const int64_t planes = zmax - zmin, min_planes = 2 * (int64_t)depth;
    if (planes < world * min_planes) return T2SC_ERR_INVALID;  // slabs too thin for the halo
    // cut points: equal voxel counts from the prefix sum of the z histogram
    // (first plane boundary whose prefix reaches total * r / world), every
    // slab at least 2 * depth planes thick
    std::vector<int64_t> cum(planes + 1, 0);
    for (int64_t r = 0; r < n; r++) cum[coords[4 * r + 3] - zmin + 1]++;
    for (int64_t i = 0; i < planes; i++) cum[i + 1] += cum[i];
    std::vector<int64_t> cuts{zmin};
    for (int r = 1; r < world; r++) {
      const double target = (double)(cum[planes] * r) / world;
      int64_t i = std::lower_bound(cum.begin(), cum.end(), target,
                                   [](int64_t v, double t) { return (double)v < t; }) -
                  cum.begin();
      i = std::max<int64_t>(i, cuts.back() - zmin + min_planes);
      i = std::min<int64_t>(i, planes - (int64_t)(world - r) * min_planes);
      cuts.push_back(zmin + i);
    }
    cuts.push_back(zmax);
    lo = cuts[rank];
    hi = cuts[rank + 1];
  }
  // local order: interior | own low band | own high band | halo below | halo above
  const bool has_lo = world > 1 && rank > 0, has_hi = world > 1 && rank < world - 1;
  std::vector<int64_t> groups[5];
  for (int64_t r = 0; r < n; r++) {
    const int64_t z = coords[4 * r + 3];
    if (z >= lo && z < hi) {
      if (has_lo && z < lo + depth)
        groups[1].push_back(r);
      else if (has_hi && z >= hi - depth)
        groups[2].push_back(r);
      else
        groups[0].push_back(r);
    } else if (has_lo && z >= lo - depth && z < lo) {
      groups[3].push_back(r);  // the lower neighbour's high band
    } else if (has_hi && z >= hi && z < hi + depth) {
      groups[4].push_back(r);  // the upper neighbour's low band
    }
  }
  const int64_t total = (int64_t)(groups[0].size() + groups[1].size() + groups[2].size() + groups[3].size() +
                                  groups[4].size());
  counts[0] = (int64_t)(groups[0].size() + groups[1].size() + groups[2].size());  // own rows
  counts[1] = (int64_t)groups[0].size();                                          // interior rows
  counts[2] = (int64_t)groups[1].size();  // sent to rank - 1
  counts[3] = (int64_t)groups[2].size();  // sent to rank + 1
  counts[4] = (int64_t)groups[3].size();  // received from rank - 1
  counts[5] = (int64_t)groups[4].size();  // received from rank + 1
  if (!rows) return T2SC_OK;
  if (total > cap) return T2SC_ERR_CAPACITY;
  int64_t o = 0;
  for (auto &g : groups)
    for (int64_t r : g) rows[o++] = r;
  return T2SC_OK;
}

int t2sc_comm_unique_id(void *id_out) {
  if (!id_out) return T2SC_ERR_INVALID;
  if (!nccl().ok) return T2SC_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (nccl().GetUniqueId(&id) != ncclSuccess) return T2SC_ERR_CUDA;
  static_assert(sizeof(ncclUniqueId) == T2SC_COMM_ID_BYTES, "NCCL unique id size");
  memcpy(id_out, &id, sizeof(id));
  return T2SC_OK;
}

int t2sc_comm_create(t2sc_ctx *ctx, const void *id, int nranks, int rank, int timeout_ms, t2sc_comm **out) {
  if (!ctx || !out || !id) return T2SC_ERR_INVALID;
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks || timeout_ms < 1)
    return fail(ctx, T2SC_ERR_INVALID, "comm: need 0 <= rank < nranks and a positive timeout");
  if (!nccl().ok) return fail(ctx, T2SC_ERR_UNSUPPORTED, "comm: libnccl.so.2 could not be loaded");
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  std::unique_ptr<t2sc_comm> c(new t2sc_comm());
  c->ctx = ctx;
  c->nranks = nranks;
  c->rank = rank;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // initialisation polled below, so a missing peer ends in a timeout
  ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  int rc = T2SC_OK;
  if (r != ncclSuccess && r != ncclInProgress) {
    rc = fail(ctx, T2SC_ERR_CUDA, nccl_msg("ncclCommInitRankConfig", r));
  } else {
    rc = wait_comm_ready(c.get(), timeout_ms, ctx->last_error);
  }
  if (prev >= 0) cudaSetDevice(prev);
  if (rc != T2SC_OK) {
    if (c->comm && !c->aborted) nccl().CommAbort(c->comm);
    return rc;
  }
  *out = c.release();
  return T2SC_OK;
}

int t2sc_comm_destroy(t2sc_comm *c) {
  if (!c) return T2SC_OK;
  if (c->comm && !c->aborted) {
    cudaStreamSynchronize(c->ctx->stream);
    // finalize flushes the communicator's work (polled, bounded: on a
    // timeout the communicator is aborted instead of destroyed)
    std::string err;
    const ncclResult_t r = nccl().CommFinalize(c->comm);
    if ((r == ncclSuccess || r == ncclInProgress) && wait_comm_ready(c, 10000, err) == T2SC_OK)
      nccl().CommDestroy(c->comm);
    else if (!c->aborted)
      nccl().CommAbort(c->comm);
  }
  delete c;
  return T2SC_OK;
}

int t2sc_comm_abort(t2sc_comm *c) {
  if (!c) return T2SC_ERR_INVALID;
  if (c->comm && !c->aborted) nccl().CommAbort(c->comm);
  c->aborted = true;
  return T2SC_OK;
}

int t2sc_halo_exchange_device(t2sc_comm *c, void *feats, int64_t row_bytes, const int64_t *counts) {
  if (!c || !counts || row_bytes <= 0) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = c->ctx;
  if (c->aborted) return fail(ctx, T2SC_ERR_INVALID, "halo exchange: the communicator was aborted");
  const int64_t n_own = counts[0], n_int = counts[1], n_lo = counts[2], n_hi = counts[3], r_lo = counts[4],
                r_hi = counts[5];
  if (n_own < 0 || n_int < 0 || n_lo < 0 || n_hi < 0 || r_lo < 0 || r_hi < 0 || n_int + n_lo + n_hi != n_own)
    return fail(ctx, T2SC_ERR_INVALID, "halo exchange: inconsistent partition counts");
  const bool lo = c->rank > 0, hi = c->rank < c->nranks - 1;
  if ((!lo && (n_lo || r_lo)) || (!hi && (n_hi || r_hi)))
    return fail(ctx, T2SC_ERR_INVALID, "halo exchange: an edge rank has rows for a missing neighbour");
  if ((n_lo + n_hi + r_lo + r_hi) > 0 && !feats) return fail(ctx, T2SC_ERR_INVALID, "halo exchange: null feats");
  uint8_t *f = static_cast<uint8_t *>(feats);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  const auto &N = nccl();
  cudaStream_t st = ctx->stream;
  ncclResult_t r = N.GroupStart();
  // rows go as bytes: the same count on both sides of every pair
  if (r == ncclSuccess && lo) {
    if (n_lo) r = N.Send(f + n_int * row_bytes, (size_t)(n_lo * row_bytes), ncclUint8, c->rank - 1, c->comm, st);
    if (r == ncclSuccess && r_lo)
      r = N.Recv(f + n_own * row_bytes, (size_t)(r_lo * row_bytes), ncclUint8, c->rank - 1, c->comm, st);
  }
  if (r == ncclSuccess && hi) {
    if (n_hi)
      r = N.Send(f + (n_int + n_lo) * row_bytes, (size_t)(n_hi * row_bytes), ncclUint8, c->rank + 1, c->comm, st);
    if (r == ncclSuccess && r_hi)
      r = N.Recv(f + (n_own + r_lo) * row_bytes, (size_t)(r_hi * row_bytes), ncclUint8, c->rank + 1, c->comm, st);
  }
  ncclResult_t r2 = N.GroupEnd();
  if (prev >= 0) cudaSetDevice(prev);
  if (r == ncclSuccess) r = r2;
  if (r == ncclInProgress) {  // non-blocking communicator: the group is still being enqueued
    return wait_comm_ready(c, 60000, ctx->last_error);
  }
  if (r != ncclSuccess) return fail(ctx, T2SC_ERR_CUDA, nccl_msg("halo exchange", r));
  return T2SC_OK;
}

int t2sc_comm_wait(t2sc_comm *c, int timeout_ms) {
  if (!c || timeout_ms < 1) return T2SC_ERR_INVALID;
  t2sc_ctx *ctx = c->ctx;
  if (c->aborted) return fail(ctx, T2SC_ERR_INVALID, "comm wait: the communicator was aborted");
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  int rc = T2SC_OK;
  for (;;) {
    cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      rc = fail(ctx, T2SC_ERR_CUDA, std::string("comm wait: ") + cudaGetErrorString(q));
      break;
    }
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      rc = fail(ctx, T2SC_ERR_CUDA, nccl_msg("comm wait", st));
      break;
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      rc = fail(ctx, T2SC_ERR_TIMEOUT, "comm wait: the stream did not drain within the timeout; communicator aborted");
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  if (prev >= 0) cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
