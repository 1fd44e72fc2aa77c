// Self-checks of two device building blocks the attention kernels rest on, each run through the
// C ABI by the library's GPU tests:
//  - the bounded mbarrier wait (ptx.cuh `mbar_wait`): a CTA waits on a barrier that nothing arms,
//    with a short limit, gives up, raises the device error word and returns, so that wavo_sync
//    reports WAVO_EDEVICE and the context stays usable;
//  - the FMA-pipe 2^x of the softmax (softmax.cuh `exp2_poly2`), evaluated over caller inputs so
//    that its error bound can be checked against exact values on the host.
#include "kernels.cuh"
#include "ptx.cuh"
#include "softmax.cuh"

namespace wv {
namespace {

// One warp waits, as the softmax warps do (mbar_wait_warp), on a barrier of one expected arrival
// that never comes. The wait ends after `limit` cycles at most: the abort is raised with the
// consumer's code and the kernel returns.
__global__ void wait_probe_kernel(int *err, long long limit) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  Abort ab{&abort_word, err};
  ab.limit = limit;
  mbar_wait_warp(&bar, 0, ab, kErrTimeoutConsumer);
  __syncthreads();
  if (threadIdx.x == 0) mbar_inval(&bar);
}

// y = 2^x by the softmax's FMA-pipe polynomial, two values a thread (the paired form it runs in).
__global__ void exp2_probe_kernel(const float *__restrict__ x, float *__restrict__ y, int n) {
  for (int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x); i < n; i += 2 * gridDim.x * blockDim.x) {
    float a = x[i], b = i + 1 < n ? x[i + 1] : 0.0f;
    exp2_poly2(a, b);
    y[i] = a;
    if (i + 1 < n) y[i + 1] = b;
  }
}

}  // namespace

cudaError_t launch_wait_probe(int *err, long long limit, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(err, limit);
  return cudaGetLastError();
}

cudaError_t launch_exp2_probe(const float *x, float *y, int n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  int blocks = (n / 2 + 255) / 256;
  if (blocks > 1184) blocks = 1184;
  exp2_probe_kernel<<<blocks, 256, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace wv
