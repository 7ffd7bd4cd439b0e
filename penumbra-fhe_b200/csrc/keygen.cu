// keygen.cu -- seeded key generation and client-side encryption on the GPU.
//
// Restates tfhe 1.6.3's gen_keys_radix (reference call site runtime/src/keys.rs:55) and
// RadixClientKey::encrypt_signed (runtime/src/encrypt.rs:21) from the published TFHE
// construction: binary secret keys, GGSW encryptions of the small-key bits under the GLWE key
// (the bootstrapping key) and LWE encryptions of the big-key bits under the small key (the
// keyswitching key).  Randomness is a ChaCha20 keystream of the caller's seed; Gaussian noise
// is Box-Muller over a series ln / cos written with explicit fma only.  This file is compiled
// with -fmad=false so that every other multiply and add rounds on its own, which makes the
// noise (and therefore every key word) reproducible bit for bit on any IEEE-754 host.
#include <cstdio>

#include "pnb_internal.cuh"
#include "pnb_keys.h"

namespace pnb {

// ln(u), u normal and > 0: u = m 2^e with m in [sqrt(1/2), sqrt(2)], ln m = 2 atanh(s),
// s = (m-1)/(m+1), atanh by its odd Taylor series to s^23.
__device__ double gauss_ln(double u) {
  const long long b = __double_as_longlong(u);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  double m = __longlong_as_double((b & 0x000fffffffffffffLL) | 0x3ff0000000000000LL);
  if (m > 0x1.6a09e667f3bcdp+0) { m = m * 0.5; e += 1; }
  const double s = (m - 1.0) / (m + 1.0);
  const double s2 = s * s;
  double p = 0x1.642c8590b2164p-5;
  p = fma(p, s2, 0x1.8618618618618p-5);
  p = fma(p, s2, 0x1.af286bca1af28p-5);
  p = fma(p, s2, 0x1.e1e1e1e1e1e1ep-5);
  p = fma(p, s2, 0x1.1111111111111p-4);
  p = fma(p, s2, 0x1.3b13b13b13b14p-4);
  p = fma(p, s2, 0x1.745d1745d1746p-4);
  p = fma(p, s2, 0x1.c71c71c71c71cp-4);
  p = fma(p, s2, 0x1.2492492492492p-3);
  p = fma(p, s2, 0x1.999999999999ap-3);
  p = fma(p, s2, 0x1.5555555555555p-2);
  p = fma(p, s2, 1.0);
  double t = s * p;
  t = t + t;
  return fma((double)e, 0x1.62e42fefa39efp-1, t);
}

// cos(2 pi u), u in [0, 1): fold to [0, 1/4], even Taylor series of cos to x^24.
__device__ double gauss_cos2pi(double u) {
  double t = u - rint(u);
  t = fabs(t);
  double sign = 1.0;
  if (t > 0.25) { t = 0.5 - t; sign = -1.0; }
  const double x = t * 0x1.921fb54442d18p+2;
  const double x2 = x * x;
  double p = 0x1.f2cf01972f578p-80;
  p = fma(p, x2, -0x1.0ce396db7f853p-70);
  p = fma(p, x2, 0x1.e542ba4020225p-62);
  p = fma(p, x2, -0x1.6827863b97d97p-53);
  p = fma(p, x2, 0x1.ae7f3e733b81fp-45);
  p = fma(p, x2, -0x1.93974a8c07c9dp-37);
  p = fma(p, x2, 0x1.1eed8eff8d898p-29);
  p = fma(p, x2, -0x1.27e4fb7789f5cp-22);
  p = fma(p, x2, 0x1.a01a01a01a01ap-16);
  p = fma(p, x2, -0x1.6c16c16c16c17p-10);
  p = fma(p, x2, 0x1.5555555555555p-5);
  p = fma(p, x2, -0.5);
  p = fma(p, x2, 1.0);
  return sign * p;
}

// Centred Gaussian of std sigma_abs (torus units), rounded to an integer; consumes keystream
// words 2*index and 2*index+1 of the noise domain.
__device__ int64_t gaussian(uint64_t seed, uint64_t domain, uint64_t index, double sigma_abs) {
  const uint64_t w1 = rand_word(seed, domain, 2 * index);
  const uint64_t w2 = rand_word(seed, domain, 2 * index + 1);
  const double u1 = (double)((w1 >> 11) + 1) * 0x1p-53;
  const double u2 = (double)(w2 >> 11) * 0x1p-53;
  const double l = gauss_ln(u1);
  const double r = sqrt(-2.0 * l);
  const double z = r * gauss_cos2pi(u2);
  const double v = z * sigma_abs;
  return (int64_t)__double2ll_rn(v);
}

__global__ void secret_keys_kernel(uint64_t* lwe_sk, int n, uint64_t* glwe_sk, int big,
                                   uint64_t seed) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) lwe_sk[i] = rand_word(seed, DOM_LWE_SK, (uint64_t)i) & 1u;
  if (i < big) glwe_sk[i] = rand_word(seed, DOM_GLWE_SK, (uint64_t)i) & 1u;
}

// Masks and noise of every GGSW row: body = e, mask c = uniform.
__global__ void bsk_fill_kernel(uint64_t* bsk, int n, int rows, int k, int N, uint64_t seed,
                                double sigma_abs) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)n * rows * N;
  if (idx >= total) return;
  const size_t g = idx / N;  // (i * rows + r)
  const int t = (int)(idx % N);
  uint64_t* row = bsk + g * (size_t)(k + 1) * N;
  row[(size_t)k * N + t] = (uint64_t)gaussian(seed, DOM_BSK_NOISE, g * N + t, sigma_abs);
  for (int c = 0; c < k; ++c)
    row[(size_t)c * N + t] = rand_word(seed, DOM_BSK_MASK, (g * k + c) * N + t);
}

// Positions of the set bits of each GLWE secret polynomial: ones[c][0..cnt[c]).
__global__ void sk_ones_kernel(const uint64_t* glwe_sk, int k, int N, int* ones, int* cnt) {
  const int c = blockIdx.x;
  if (c >= k || threadIdx.x != 0) return;
  int m = 0;
  for (int j = 0; j < N; ++j)
    if (glwe_sk[(size_t)c * N + j]) ones[(size_t)c * N + m++] = j;
  cnt[c] = m;
}

// body += sum_c A_c * S_c (negacyclic, S binary), then the gadget term on row (comp, lev).
// One block per GGSW row; the secret key enters as the list of its set positions.
template <int PER>
__global__ void __launch_bounds__(256) bsk_body_kernel(uint64_t* bsk, const int* ones_g,
                                                       const int* cnt_g,
                                                       const uint64_t* lwe_sk, int rows, int k,
                                                       int N, int level, int base_log) {
  extern __shared__ uint64_t bsm[];
  uint64_t* A = bsm;                            // N words
  int* ones = reinterpret_cast<int*>(bsm + N);  // up to N indices
  const size_t g = blockIdx.x;
  const int i = (int)(g / rows), r = (int)(g % rows);
  uint64_t* row = bsk + g * (size_t)(k + 1) * N;
  uint64_t* body = row + (size_t)k * N;
  uint64_t acc[PER];  // outputs per thread: N <= 256 PER
  const int per = (N + blockDim.x - 1) / blockDim.x;
#pragma unroll
  for (int q = 0; q < PER; ++q) acc[q] = 0;
  for (int c = 0; c < k; ++c) {
    __syncthreads();
    const int cnt = cnt_g[c];
    for (int t = threadIdx.x; t < N; t += blockDim.x) {
      A[t] = row[(size_t)c * N + t];
      ones[t] = ones_g[(size_t)c * N + t];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int t = threadIdx.x + q * blockDim.x;
      if (q < per && t < N) {
        uint64_t s = 0;
        for (int e = 0; e < cnt; ++e) {
          const int src = t - ones[e];
          s += (src >= 0) ? A[src] : (uint64_t)0 - A[src + N];
        }
        acc[q] += s;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int t = threadIdx.x + q * blockDim.x;
    if (q < per && t < N) body[t] += acc[q];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int comp = r / level, lev = r % level;
    row[(size_t)comp * N] += lwe_sk[i] << (64 - base_log * (lev + 1));
  }
}

// One block per keyswitching-key row (i, j): LWE encryption of S_big[i] * q / B^(j+1).
__global__ void __launch_bounds__(128) ksk_kernel(uint64_t* ksk, const uint64_t* glwe_sk,
                                                  const uint64_t* lwe_sk, int n, int row_words,
                                                  int level, int base_log, uint64_t seed,
                                                  double sigma_abs) {
  __shared__ uint64_t red[128];
  const size_t rowi = blockIdx.x;  // i * level + j
  const int i = (int)(rowi / level), j = (int)(rowi % level);
  uint64_t* ct = ksk + rowi * (size_t)row_words;
  for (int t = n + 1 + threadIdx.x; t < row_words; t += 128) ct[t] = 0;  // row padding
  uint64_t part = 0;
  for (int t = threadIdx.x; t < n; t += 128) {
    const uint64_t a = rand_word(seed, DOM_KSK_MASK, rowi * n + t);
    ct[t] = a;
    part += a * lwe_sk[t];
  }
  red[threadIdx.x] = part;
  __syncthreads();
  for (int s = 64; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    uint64_t b = red[0];
    b += (uint64_t)gaussian(seed, DOM_KSK_NOISE, rowi, sigma_abs);
    b += glwe_sk[i] << (64 - base_log * (j + 1));
    ct[n] = b;
  }
}

// Client-side LWE encryption under a key of dimension `dim`: one block per ciphertext.
__global__ void __launch_bounds__(256) encrypt_kernel(const int64_t* msg, uint64_t delta,
                                                      uint64_t seed, uint64_t first,
                                                      const uint64_t* key, int dim,
                                                      double sigma_abs, uint64_t* ct_out) {
  __shared__ uint64_t red[256];
  const uint64_t index = first + blockIdx.x;
  uint64_t* ct = ct_out + (size_t)blockIdx.x * (dim + 1);
  uint64_t part = 0;
  for (int t = threadIdx.x; t < dim; t += 256) {
    const uint64_t a = rand_word(seed, DOM_ENC_MASK, index * (uint64_t)dim + t);
    ct[t] = a;
    part += a * key[t];
  }
  red[threadIdx.x] = part;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    uint64_t b = red[0] + (uint64_t)gaussian(seed, DOM_ENC_NOISE, index, sigma_abs);
    ct[dim] = b + (uint64_t)msg[blockIdx.x] * delta;
  }
}

int keygen_device(pnb_keys* K, cudaStream_t st) {
  const pnb_params& p = K->p;
  const int big = p.k * p.N, rows = (p.k + 1) * p.pbs_level;
  const int nmax = big > p.n ? big : p.n;
  if (p.N > 8192) {
    set_error("keygen: the bootstrapping-key body kernel covers N <= 8192 (got %d)", p.N);
    return PNB_ERR_UNSUPPORTED;
  }
  secret_keys_kernel<<<(nmax + 255) / 256, 256, 0, st>>>(K->lwe_sk, p.n, K->glwe_sk, big,
                                                           K->seed);
  PNB_CHECK_LAUNCH("secret_keys_kernel");
  const size_t fill = (size_t)p.n * rows * p.N;
  bsk_fill_kernel<<<(unsigned)((fill + 255) / 256), 256, 0, st>>>(
      K->bsk, p.n, rows, p.k, p.N, K->seed, p.glwe_std * 0x1p64);
  PNB_CHECK_LAUNCH("bsk_fill_kernel");
  int* ones = nullptr;
  PNB_CUDA(cudaMallocAsync((void**)&ones, sizeof(int) * ((size_t)p.k * p.N + p.k), st));
  sk_ones_kernel<<<p.k, 32, 0, st>>>(K->glwe_sk, p.k, p.N, ones, ones + (size_t)p.k * p.N);
  PNB_CHECK_LAUNCH("sk_ones_kernel");
  const int smem = p.N * (int)sizeof(uint64_t) + p.N * (int)sizeof(int);
  if (p.N <= 4096) {
    PNB_CUDA(cudaFuncSetAttribute(bsk_body_kernel<16>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    bsk_body_kernel<16><<<p.n * rows, 256, smem, st>>>(K->bsk, ones, ones + (size_t)p.k * p.N,
                                                       K->lwe_sk, rows, p.k, p.N, p.pbs_level,
                                                       p.pbs_base_log);
  } else {
    PNB_CUDA(cudaFuncSetAttribute(bsk_body_kernel<32>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    bsk_body_kernel<32><<<p.n * rows, 256, smem, st>>>(K->bsk, ones, ones + (size_t)p.k * p.N,
                                                       K->lwe_sk, rows, p.k, p.N, p.pbs_level,
                                                       p.pbs_base_log);
  }
  PNB_CHECK_LAUNCH("bsk_body_kernel");
  PNB_CUDA(cudaFreeAsync(ones, st));
  ksk_kernel<<<big * p.ks_level, 128, 0, st>>>(K->ksk, K->glwe_sk, K->lwe_sk, p.n, K->ksk_row,
                                               p.ks_level, p.ks_base_log, K->seed,
                                               p.lwe_std * 0x1p64);
  PNB_CHECK_LAUNCH("ksk_kernel");
  return PNB_OK;
}

int encrypt_lwe(const pnb_keys* K, const int64_t* msg, uint64_t delta, uint64_t seed,
                uint64_t first, uint64_t* ct, int count, cudaStream_t st) {
  if (count <= 0) return PNB_OK;
  const int big = K->p.k * K->p.N;
  encrypt_kernel<<<count, 256, 0, st>>>(msg, delta, seed, first, K->glwe_sk, big,
                                        K->p.glwe_std * 0x1p64, ct);
  PNB_CHECK_LAUNCH("encrypt_kernel");
  return PNB_OK;
}

}  // namespace pnb
