// lwe.cu -- LWE phase (client decrypt), the ciphertext x cleartext-weight contraction, and the
// FP64 throughput probe used as the blind rotation's roofline denominator.
#include <cstdio>

#include "pnb_internal.cuh"
#include "pnb_keys.h"

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
// Contraction Y[b][j][c] = sum_i W[j][i] X[b][i][c] (+ bias[j]*delta on the body column).
// CUDA-core version: a block owns (sample b, 32 output rows, 256 columns); each thread owns
// one column and 32 row accumulators; W rows of the tile are staged in shared memory.
// ------------------------------------------------------------------------------------------
constexpr int CT_ROWS = 32;
constexpr int CT_COLS = 256;
constexpr int CT_KCH = 64;

__global__ void __launch_bounds__(CT_COLS) contract_kernel(
    const int8_t* __restrict__ W, const int64_t* __restrict__ bias, uint64_t delta, int M, int K,
    const uint64_t* __restrict__ X, uint64_t* __restrict__ Y, int lwe_len) {
  __shared__ int32_t ws[CT_ROWS][CT_KCH];
  const int b = blockIdx.z;
  const int j0 = blockIdx.y * CT_ROWS;
  const int c = blockIdx.x * CT_COLS + threadIdx.x;
  const int rows = min(CT_ROWS, M - j0);
  uint64_t acc[CT_ROWS];
#pragma unroll
  for (int r = 0; r < CT_ROWS; ++r) acc[r] = 0;
  const uint64_t* xb = X + (size_t)b * K * lwe_len;
  for (int k0 = 0; k0 < K; k0 += CT_KCH) {
    __syncthreads();
    for (int e = threadIdx.x; e < CT_ROWS * CT_KCH; e += CT_COLS) {
      const int r = e / CT_KCH, kk = e % CT_KCH;
      ws[r][kk] = (r < rows && k0 + kk < K) ? (int32_t)W[(size_t)(j0 + r) * K + k0 + kk] : 0;
    }
    __syncthreads();
    if (c < lwe_len) {
      const int kmax = min(CT_KCH, K - k0);
      for (int kk = 0; kk < kmax; ++kk) {
        const uint64_t x = __ldg(xb + (size_t)(k0 + kk) * lwe_len + c);
#pragma unroll
        for (int r = 0; r < CT_ROWS; ++r) acc[r] += (uint64_t)(int64_t)ws[r][kk] * x;
      }
    }
  }
  if (c < lwe_len) {
#pragma unroll
    for (int r = 0; r < CT_ROWS; ++r) {
      if (r < rows) {
        uint64_t v = acc[r];
        if (bias && c == lwe_len - 1) v += (uint64_t)bias[j0 + r] * delta;
        Y[((size_t)b * M + j0 + r) * lwe_len + c] = v;
      }
    }
  }
}

int lwe_contract(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                 const uint64_t* X, uint64_t* Y, int batch, int lwe_len, cudaStream_t st) {
  if (M <= 0 || K <= 0 || batch < 0 || lwe_len <= 0) {
    set_error("lwe_contract: bad shape M=%d K=%d batch=%d lwe_len=%d", M, K, batch, lwe_len);
    return PNB_ERR_INVALID;
  }
  if (batch == 0) return PNB_OK;
  if (batch > 65535) {
    set_error("lwe_contract: batch %d exceeds the grid limit of 65535 per call", batch);
    return PNB_ERR_INVALID;
  }
  dim3 grid((lwe_len + CT_COLS - 1) / CT_COLS, (M + CT_ROWS - 1) / CT_ROWS, batch);
  contract_kernel<<<grid, CT_COLS, 0, st>>>(W, bias, delta, M, K, X, Y, lwe_len);
  PNB_CHECK_LAUNCH("contract_kernel");
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

}  // namespace pnb
