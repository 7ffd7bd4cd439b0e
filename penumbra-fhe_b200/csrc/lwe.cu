// lwe.cu -- LWE phase (client decrypt) and the FP64 throughput probe used as the blind
// rotation's roofline denominator.  (The contraction is in contract_tc.cu.)
#include <cstdio>

#include "pnb_internal.cuh"
#include "pnb_keys.h"
#include "tc_primitives.cuh"

namespace pnb {

// Phase b - <a, s>: one warp per ciphertext.
__global__ void phase_kernel(const uint64_t* __restrict__ ct, const uint64_t* __restrict__ key,
                             int dim, uint64_t* __restrict__ phase, int count) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= count) return;
  const uint64_t* c = ct + (size_t)w * (dim + 1);
  uint64_t s = 0;
  for (int t = lane; t < dim; t += 32) s += c[t] * key[t];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) phase[w] = c[dim] - s;
}

int phase_lwe(const pnb_keys* K, const uint64_t* ct, uint64_t* phase, int count, int small,
              cudaStream_t st) {
  if (count <= 0) return PNB_OK;
  const int dim = small ? K->p.n : K->p.k * K->p.N;
  const uint64_t* key = small ? K->lwe_sk : K->glwe_sk;
  phase_kernel<<<(count + 7) / 8, 256, 0, st>>>(ct, key, dim, phase, count);
  PNB_CHECK_LAUNCH("phase_kernel");
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// FP64 FMA throughput probe: 8 independent FMA chains per thread, registers only.
// ------------------------------------------------------------------------------------------
__global__ void fp64_probe_kernel(double* out, int iters, double a, double b) {
  double x0 = threadIdx.x * 1e-9, x1 = x0 + 1, x2 = x0 + 2, x3 = x0 + 3;
  double x4 = x0 + 4, x5 = x0 + 5, x6 = x0 + 6, x7 = x0 + 7;
  for (int i = 0; i < iters; ++i) {
    x0 = fma(x0, a, b); x1 = fma(x1, a, b); x2 = fma(x2, a, b); x3 = fma(x3, a, b);
    x4 = fma(x4, a, b); x5 = fma(x5, a, b); x6 = fma(x6, a, b); x7 = fma(x7, a, b);
  }
  out[blockIdx.x * blockDim.x + threadIdx.x] = x0 + x1 + x2 + x3 + x4 + x5 + x6 + x7;
}

int measure_fp64_peak(double* tflops) {
  int dev = 0, sms = 0;
  PNB_CUDA(cudaGetDevice(&dev));
  PNB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int blocks = sms * 8, threads = 256, iters = 20000;
  double* d = nullptr;
  PNB_CUDA(cudaMalloc(&d, sizeof(double) * blocks * threads));
  cudaEvent_t e0, e1;
  PNB_CUDA(cudaEventCreate(&e0));
  PNB_CUDA(cudaEventCreate(&e1));
  float best = 1e30f;
  for (int rep = 0; rep < 4; ++rep) {
    PNB_CUDA(cudaEventRecord(e0, 0));
    fp64_probe_kernel<<<blocks, threads>>>(d, iters, 0.999999, 1e-7);
    PNB_CUDA(cudaEventRecord(e1, 0));
    PNB_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    PNB_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    if (rep > 0 && ms < best) best = ms;
  }
  PNB_CUDA(cudaEventDestroy(e0));
  PNB_CUDA(cudaEventDestroy(e1));
  PNB_CUDA(cudaFree(d));
  const double flops = 2.0 * 8 * (double)iters * blocks * threads;
  *tflops = flops / (best * 1e-3) / 1e12;
  return PNB_OK;
}

// The bounded mbarrier wait of the rotation, keyswitch and contraction kernels, run against a
// barrier that nothing completes: every thread gives up after `polls` polls and the block
// records that it did.  Nothing is in flight on the barrier, so the block exits cleanly and the
// context stays usable -- the property the real kernels rely on when a copy never lands.
__global__ void wait_probe_kernel(uint32_t polls, int* gave_up) {
  __shared__ __align__(8) uint64_t bar_word;
  const uint32_t bar = tc::smem_u32(&bar_word);
  if (threadIdx.x == 0) {
    tc::mbar_init(bar, 1);  // one arrival expected, none ever made
    tc::fence_mbar_init();
  }
  __syncthreads();
  const bool done = tc::mbar_wait(bar, 0u, polls);
  if (!__all_sync(0xffffffffu, done) && (threadIdx.x & 31) == 0) atomicAdd(gave_up, 1);
}

int wait_probe(uint32_t polls, int* warps_gave_up) {
  int* d = nullptr;
  PNB_CUDA(cudaMalloc(&d, sizeof(int)));
  PNB_CUDA(cudaMemset(d, 0, sizeof(int)));
  wait_probe_kernel<<<1, 64>>>(polls, d);
  PNB_CHECK_LAUNCH("wait_probe_kernel");
  PNB_CUDA(cudaMemcpy(warps_gave_up, d, sizeof(int), cudaMemcpyDeviceToHost));
  PNB_CUDA(cudaFree(d));
  return PNB_OK;
}

}  // namespace pnb
