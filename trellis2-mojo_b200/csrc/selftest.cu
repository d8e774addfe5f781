// Device self-test (the reference runs one when it opens its GPU context,
// trellis2_mojo/gpu/context.mojo:7-12, 139-158): a small compute check, and
// a check of the bounded-wait path every conv pipeline relies on. The
// second part waits on an mbarrier that nothing completes, with a short
// limit, and must come back with the timeout flag set instead of hanging.
#include "internal.h"
#include "sm100.cuh"

namespace t2sc {
namespace {

__global__ void selftest_kernel(const float *__restrict__ in, float *__restrict__ out, int n, long long wait_cycles,
                                int *flags) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = in[i] * 2.0f + 1.0f;
  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(&bar), 1);
    abort_flag = 0;
    sm100::fence_mbar_init();
    // phase 0 never completes: no thread arrives
    const bool ok = sm100::mbar_wait_bounded(sm100::smem_u32(&bar), 0, &abort_flag, flags, kDevErrTimeout,
                                             wait_cycles);
    if (ok) atomicOr(flags, kDevErrInternal);  // a wait that nothing can satisfy returned success
  }
}

}  // namespace
}  // namespace t2sc

using namespace t2sc;

extern "C" int t2sc_ctx_selftest(t2sc_ctx *ctx, int wait_us) {
  if (!ctx) return T2SC_ERR_INVALID;
  std::string &err = ctx->last_error;
  if (wait_us < 1 || wait_us > 1000000) {
    err = "selftest: wait_us must be in [1, 1000000]";
    return T2SC_ERR_INVALID;
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  int rc = [&]() -> int {
    const int n = 256;
    float h_in[n], h_out[n];
    for (int i = 0; i < n; i++) h_in[i] = (float)i - 100.0f;
    float *d = nullptr;
    int *d_flags = nullptr;
    T2SC_CUDA(cudaMalloc((void **)&d, 2 * n * sizeof(float)), "selftest buffers");
    T2SC_CUDA(cudaMalloc((void **)&d_flags, sizeof(int)), "selftest flags");
    int r = T2SC_OK;
    int h_flags = 0;
    do {
      if ((r = cuda_status(cudaMemcpy(d, h_in, n * sizeof(float), cudaMemcpyHostToDevice), err, "selftest")) != T2SC_OK) break;
      if ((r = cuda_status(cudaMemset(d_flags, 0, sizeof(int)), err, "selftest")) != T2SC_OK) break;
      // the SM clock is at most ~2 GHz: 2000 cycles per microsecond
      selftest_kernel<<<1, 64, 0, ctx->stream>>>(d, d + n, n, 2000LL * wait_us, d_flags);
      ctx->launches++;
      if ((r = cuda_status(cudaGetLastError(), err, "selftest launch")) != T2SC_OK) break;
      if ((r = cuda_status(cudaStreamSynchronize(ctx->stream), err, "selftest")) != T2SC_OK) break;
      if ((r = cuda_status(cudaMemcpy(h_out, d + n, n * sizeof(float), cudaMemcpyDeviceToHost), err, "selftest")) != T2SC_OK) break;
      if ((r = cuda_status(cudaMemcpy(&h_flags, d_flags, sizeof(int), cudaMemcpyDeviceToHost), err, "selftest")) != T2SC_OK) break;
      for (int i = 0; i < n; i++)
        if (h_out[i] != h_in[i] * 2.0f + 1.0f) {
          err = "selftest: compute check failed";
          r = T2SC_ERR_CUDA;
          break;
        }
      if (r != T2SC_OK) break;
      if (!(h_flags & kDevErrTimeout) || (h_flags & kDevErrInternal)) {
        err = "selftest: the bounded wait did not report its timeout";
        r = T2SC_ERR_CUDA;
      }
    } while (0);
    cudaFree(d);
    cudaFree(d_flags);
    return r;
  }();
  int cur = -1;
  if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  return rc;
}
