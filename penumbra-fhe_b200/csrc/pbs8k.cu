// pbs8k.cu -- blind rotation and Fourier key conversion at polynomial size N = 8192 (k = 1).
//
// The same bootstrap as pbs.cu (keyswitch, modulus switch to 2N, blind rotation through GGSW x
// GLWE external products in the f64 Fourier domain, sample extraction of coefficient 0), for the
// 6-bit parameter set whose GLWE polynomials have 8192 coefficients.  A polynomial folds into
// M = 4096 complex points y_j = a_j + i a_{j+M}, evaluated at the M roots of X^M = i (the
// evaluation tfhe-rs performs with its f64 FFT, restated here for a 256-thread transform):
//
//   thread t holds y_{t + 256 m} for m = 0..15 (the "natural" distribution);
//   pass 1: multiply by c_m = exp(i pi m / 32), DFT16 over m, multiply output k1 by
//           exp(i pi t (1 + 4 k1) / 8192) (the negacyclic twist and the first twiddle in one),
//           transpose through shared memory;
//   pass 2: thread (k1, j4) takes t = 16 j3 + j4 for j3 = 0..15: DFT16 over j3, multiply output
//           k3 by exp(2 pi i j4 k3 / 256), transpose;
//   pass 3: thread (k1, k3) takes j4 = 0..15: DFT16 over j4.
// Register k4 of thread v = 16 k1 + k3 then holds y(zeta w^K), K = k1 + 16 k3 + 256 k4,
// zeta = exp(i pi / 8192), w = exp(2 pi i / 4096): the "spectral" distribution, in which the
// Fourier bootstrapping key is stored ([k4][v], so every key read is coalesced).  The inverse
// runs the three passes backwards with conjugate factors and a 2^-12 scale.
//
// Rotation: one ciphertext per block of 256 threads.  The accumulator (top 32 bits of each torus
// coefficient, coefficients j and j + M side by side) sits in shared memory with one 64 KB
// transpose buffer; per CMux every (row, level) digit polynomial is transformed and multiplied
// into both output spectra, which stay in registers until their inverse transforms.  One GGSW
// row (two output polynomials, 128 KB) does not fit shared memory beside the transpose buffer and
// the accumulator, so the key streams through a ring of 32 KB stages filled by bulk copies
// (cp.async.bulk, no multicast) one step ahead of the products: while a row's digits are formed
// and transformed, the first stages of its key land.  The transform's twiddle tables sit in
// tensor memory (each warp's threads' factors in its lane quarter), not behind L1.
#include <cmath>
#include <mutex>
#include <vector>

#include "fft1024.cuh"
#include "pnb_internal.cuh"
#include "pnb_keys.h"
#include "tc_primitives.cuh"

namespace pnb {

constexpr int N8 = 8192, M8 = 4096, T8 = 256;  // polynomial size, points, threads
constexpr int BR8_MAXN = 1024;                  // small LWE dimension the shared layout holds

// Device-side status word of the N = 8192 rotation: non-zero when a bounded wait ran out.
__device__ int g_br8_status;

int br8_status_read_and_clear(int* out) {
  int v = 0;
  PNB_CUDA(cudaMemcpyFromSymbol(&v, g_br8_status, sizeof(int)));
  const int zero = 0;
  PNB_CUDA(cudaMemcpyToSymbol(g_br8_status, &zero, sizeof(int)));
  *out = v;
  return PNB_OK;
}

// ---- tables (one set per device) -----------------------------------------------------------
struct Fft8Tables {
  double2* tw1;  // [k1][t]: exp(i pi t (1 + 4 k1) / 8192), k1 < 16, t < 256
  double2* tw2;  // [k3][j4]: exp(2 pi i j4 k3 / 256)
  double2* cm;   // [m]: exp(i pi m / 32)
};

static std::mutex g_t8_mu;
static Fft8Tables g_t8[64];
static bool g_t8_ok[64];

static double2 cis_pi(long long num, long long den) {  // exp(i pi num / den)
  const long double PI = 3.141592653589793238462643383279502884L;
  const long long e = ((num % (2 * den)) + 2 * den) % (2 * den);
  const long double a = PI * (long double)e / (long double)den;
  return make_double2((double)cosl(a), (double)sinl(a));
}

static int fft8_tables_get(Fft8Tables* out) {
  int dev = 0;
  PNB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("device index %d out of range", dev);
    return PNB_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_t8_mu);
  if (!g_t8_ok[dev]) {
    std::vector<double2> a(16 * T8), b(256), c(16);
    for (int k1 = 0; k1 < 16; ++k1)
      for (int t = 0; t < T8; ++t) a[k1 * T8 + t] = cis_pi((long long)t * (1 + 4 * k1), 8192);
    for (int k3 = 0; k3 < 16; ++k3)
      for (int j4 = 0; j4 < 16; ++j4) b[k3 * 16 + j4] = cis_pi(2LL * j4 * k3, 256);
    for (int m = 0; m < 16; ++m) c[m] = cis_pi(m, 32);
    Fft8Tables t{};
    PNB_CUDA(cudaMalloc(&t.tw1, sizeof(double2) * a.size()));
    PNB_CUDA(cudaMalloc(&t.tw2, sizeof(double2) * b.size()));
    PNB_CUDA(cudaMalloc(&t.cm, sizeof(double2) * c.size()));
    PNB_CUDA(cudaMemcpy(t.tw1, a.data(), sizeof(double2) * a.size(), cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.tw2, b.data(), sizeof(double2) * b.size(), cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.cm, c.data(), sizeof(double2) * c.size(), cudaMemcpyHostToDevice));
    g_t8[dev] = t;
    g_t8_ok[dev] = true;
  }
  *out = g_t8[dev];
  return PNB_OK;
}

// ---- the transform ---------------------------------------------------------------------------
// out_k = sum_m in_m exp(S 2 pi i m k / 16), natural order in and out: a bit-reversal in
// registers, then decimation-in-time stages whose butterflies are pnb::ct_bfly's
// (u, v) <- (u + w v, u - w v), w = exp(2 pi i e / 128).
template <int S, int L>
__device__ __forceinline__ void dit16_stage(double2 (&x)[16]) {
#pragma unroll
  for (int s = 0; s < 16; s += L) {
#pragma unroll
    for (int j = 0; j < L / 2; ++j) {
      constexpr int sign = S > 0 ? 1 : -1;
      ct_bfly<true>((sign * 128 * j / L) & 127, x[s + j], x[s + j + L / 2]);
    }
  }
}

template <int S>
__device__ __forceinline__ void dft16(double2 (&x)[16]) {
  // bit-reversal permutation: swap the pairs (1,8) (2,4) (3,12) (5,10) (7,14) (11,13)
  auto sw = [&](int a, int b) {
    const double2 t = x[a];
    x[a] = x[b];
    x[b] = t;
  };
  sw(1, 8); sw(2, 4); sw(3, 12); sw(5, 10); sw(7, 14); sw(11, 13);
  dit16_stage<S, 2>(x);
  dit16_stage<S, 4>(x);
  dit16_stage<S, 8>(x);
  dit16_stage<S, 16>(x);
}

__device__ __forceinline__ int swz8(int row, int col) { return row * 16 + (col ^ (row & 7)); }

__device__ __forceinline__ double2 conjd(double2 v) { return make_double2(v.x, -v.y); }

// Natural -> spectral distribution (thread t = threadIdx.x of 256); buf is 4096 double2.
__device__ __forceinline__ void fwd8k(double2 (&x)[16], double2* buf, const Fft8Tables& tb) {
  const int t = threadIdx.x;
#pragma unroll
  for (int m = 0; m < 16; ++m) x[m] = cmul(x[m], __ldg(&tb.cm[m]));
  dft16<1>(x);
#pragma unroll
  for (int k1 = 0; k1 < 16; ++k1) x[k1] = cmul(x[k1], __ldg(&tb.tw1[k1 * T8 + t]));
#pragma unroll
  for (int k1 = 0; k1 < 16; ++k1) buf[swz8(t, k1)] = x[k1];
  __syncthreads();
  const int k1 = t >> 4, j4 = t & 15;
#pragma unroll
  for (int j3 = 0; j3 < 16; ++j3) x[j3] = buf[swz8(16 * j3 + j4, k1)];
  __syncthreads();
  dft16<1>(x);
#pragma unroll
  for (int k3 = 0; k3 < 16; ++k3) x[k3] = cmul(x[k3], __ldg(&tb.tw2[k3 * 16 + j4]));
#pragma unroll
  for (int k3 = 0; k3 < 16; ++k3) buf[swz8(16 * k1 + j4, k3)] = x[k3];
  __syncthreads();
  const int k3 = t & 15;  // thread v = 16 k1 + k3 (same t)
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = buf[swz8(16 * k1 + q, k3)];
  __syncthreads();
  dft16<1>(x);
}

// Spectral -> natural distribution, scaled by 2^-12 * `scale` (a power of two).
__device__ __forceinline__ void inv8k(double2 (&x)[16], double2* buf, const Fft8Tables& tb,
                                      double scale) {
  const int t = threadIdx.x;
  const int k1 = t >> 4, k3 = t & 15;
  dft16<-1>(x);  // over k4 -> j4
#pragma unroll
  for (int j4 = 0; j4 < 16; ++j4) buf[swz8(16 * k1 + j4, k3)] = x[j4];
  __syncthreads();
  const int j4 = t & 15;  // thread u = 16 k1 + j4
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = cmul(buf[swz8(16 * k1 + j4, q)], conjd(__ldg(&tb.tw2[q * 16 + j4])));
  __syncthreads();
  dft16<-1>(x);  // over k3 -> j3
#pragma unroll
  for (int j3 = 0; j3 < 16; ++j3) buf[swz8(16 * j3 + j4, k1)] = x[j3];
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = cmul(buf[swz8(t, q)], conjd(__ldg(&tb.tw1[q * T8 + t])));
  __syncthreads();
  dft16<-1>(x);  // over k1 -> m
  const double sc = scale * (1.0 / 4096.0);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const double2 c = __ldg(&tb.cm[m]);
    x[m] = cmul(x[m], make_double2(c.x * sc, -c.y * sc));
  }
}

// The rotation's transforms take the twiddle factors of this thread from tensor memory: per
// warp, columns [0, 64) hold tw1[k1][t] for k1 = 0..15 and [64, 128) hold tw2[k3][t & 15] for
// k3 = 0..15, each complex value as four 32-bit words (re lo, re hi, im lo, im hi).
__device__ __forceinline__ void tw_words(double2 v, uint32_t* w) {
  w[0] = (uint32_t)__double2loint(v.x);
  w[1] = (uint32_t)__double2hiint(v.x);
  w[2] = (uint32_t)__double2loint(v.y);
  w[3] = (uint32_t)__double2hiint(v.y);
}
__device__ __forceinline__ double2 spec_of_words(const uint32_t* w) {
  return make_double2(__hiloint2double((int)w[1], (int)w[0]), __hiloint2double((int)w[3], (int)w[2]));
}

// x[q] *= T[q] (CONJ: by conj(T[q])) for the 16 factors at tensor-memory address `ta`.
#ifndef PNB_BR8_TW_CHUNK
#define PNB_BR8_TW_CHUNK 4  // complex factors per tensor-memory load (4: 16 columns, 8: 32)
#endif
__device__ __forceinline__ void tm_words(uint32_t ta, uint32_t (&w)[16]) {
  tc::tmem_ld_32x32_x16(ta, w);
}
__device__ __forceinline__ void tm_words(uint32_t ta, uint32_t (&w)[32]) {
  tc::tmem_ld_32x32_nowait(ta, w);
}
template <bool CONJ>
__device__ __forceinline__ void tm_twiddle16(double2 (&x)[16], uint32_t ta) {
  constexpr int C = PNB_BR8_TW_CHUNK;
  static_assert(C == 4 || C == 8, "4 or 8 factors per load");
#pragma unroll
  for (int g = 0; g < 16 / C; ++g) {
    uint32_t w[4 * C];
    tm_words(ta + 4u * C * g, w);
    tc::tmem_ld_wait();
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const double2 c = make_double2(__hiloint2double((int)w[4 * q + 1], (int)w[4 * q]),
                                     __hiloint2double((int)w[4 * q + 3], (int)w[4 * q + 2]));
      x[C * g + q] = CONJ ? cmul_conj(x[C * g + q], c) : cmul(x[C * g + q], c);
    }
  }
}

// fwd8k with the twiddles from tensor memory (t_tw1, t_tw2: this warp's column bases).
__device__ __forceinline__ void fwd8k_tm(double2 (&x)[16], double2* buf, const Fft8Tables& tb,
                                         uint32_t t_tw1, uint32_t t_tw2) {
  const int t = threadIdx.x;
#pragma unroll
  for (int m = 0; m < 16; ++m) x[m] = cmul(x[m], __ldg(&tb.cm[m]));
  dft16<1>(x);
  tm_twiddle16<false>(x, t_tw1);
#pragma unroll
  for (int k1 = 0; k1 < 16; ++k1) buf[swz8(t, k1)] = x[k1];
  __syncthreads();
  const int k1 = t >> 4, j4 = t & 15;
#pragma unroll
  for (int j3 = 0; j3 < 16; ++j3) x[j3] = buf[swz8(16 * j3 + j4, k1)];
  __syncthreads();
  dft16<1>(x);
  tm_twiddle16<false>(x, t_tw2);
#pragma unroll
  for (int k3 = 0; k3 < 16; ++k3) buf[swz8(16 * k1 + j4, k3)] = x[k3];
  __syncthreads();
  const int k3 = t & 15;
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = buf[swz8(16 * k1 + q, k3)];
  __syncthreads();
  dft16<1>(x);
}

// inv8k with the twiddles from tensor memory.
__device__ __forceinline__ void inv8k_tm(double2 (&x)[16], double2* buf, const Fft8Tables& tb,
                                         uint32_t t_tw1, uint32_t t_tw2, double scale) {
  const int t = threadIdx.x;
  const int k1 = t >> 4, k3 = t & 15;
  dft16<-1>(x);
#pragma unroll
  for (int j4 = 0; j4 < 16; ++j4) buf[swz8(16 * k1 + j4, k3)] = x[j4];
  __syncthreads();
  const int j4 = t & 15;
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = buf[swz8(16 * k1 + j4, q)];
  __syncthreads();
  tm_twiddle16<true>(x, t_tw2);
  dft16<-1>(x);
#pragma unroll
  for (int j3 = 0; j3 < 16; ++j3) buf[swz8(16 * j3 + j4, k1)] = x[j3];
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = buf[swz8(t, q)];
  __syncthreads();
  tm_twiddle16<true>(x, t_tw1);
  dft16<-1>(x);
  const double sc = scale * (1.0 / 4096.0);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const double2 c = __ldg(&tb.cm[m]);
    x[m] = cmul(x[m], make_double2(c.x * sc, -c.y * sc));
  }
}

// ---- Fourier conversion of the bootstrapping key ------------------------------------------
__global__ void __launch_bounds__(T8) bsk8k_to_fourier_kernel(const uint64_t* __restrict__ bsk,
                                                              double2* __restrict__ fbsk,
                                                              Fft8Tables tb) {
  extern __shared__ double2 f8buf[];
  const size_t poly = blockIdx.x;
  const uint64_t* a = bsk + poly * N8;
  const int t = threadIdx.x;
  double2 x[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = t + T8 * m;
    x[m] = make_double2(__ll2double_rn((long long)a[j]), __ll2double_rn((long long)a[j + M8]));
  }
  fwd8k(x, f8buf, tb);
  double2* o = fbsk + poly * M8;
#pragma unroll
  for (int q = 0; q < 16; ++q) o[q * T8 + t] = x[q];
}

int bsk_to_fourier_8k(const uint64_t* bsk_dev, double2* fbsk_dev, int polys, cudaStream_t st) {
  Fft8Tables tb;
  int rc = fft8_tables_get(&tb);
  if (rc) return rc;
  const int smem = M8 * sizeof(double2);
  PNB_CUDA(cudaFuncSetAttribute(bsk8k_to_fourier_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  bsk8k_to_fourier_kernel<<<polys, T8, smem, st>>>(bsk_dev, fbsk_dev, tb);
  PNB_CHECK_LAUNCH("bsk8k_to_fourier_kernel");
  return PNB_OK;
}

// ---- diagnostic: negacyclic products through the transform -------------------------------------
__global__ void __launch_bounds__(T8) fft8k_mul_kernel(const int64_t* __restrict__ a,
                                                       const uint64_t* __restrict__ b,
                                                       uint64_t* __restrict__ out, Fft8Tables tb) {
  extern __shared__ double2 m8buf[];
  const size_t poly = blockIdx.x;
  const int t = threadIdx.x;
  double2 x[16], y[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = t + T8 * m;
    x[m] = make_double2(__ll2double_rn(a[poly * N8 + j]), __ll2double_rn(a[poly * N8 + j + M8]));
  }
  fwd8k(x, m8buf, tb);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = t + T8 * m;
    y[m] = make_double2(__ll2double_rn((long long)b[poly * N8 + j]),
                        __ll2double_rn((long long)b[poly * N8 + j + M8]));
  }
  fwd8k(y, m8buf, tb);
#pragma unroll
  for (int q = 0; q < 16; ++q) x[q] = cmul(x[q], y[q]);
  inv8k(x, m8buf, tb, 1.0);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = t + T8 * m;
    out[poly * N8 + j] = f64_to_torus(x[m].x);
    out[poly * N8 + j + M8] = f64_to_torus(x[m].y);
  }
}

int fft_negacyclic_mul_8k(const int64_t* a, const uint64_t* b, uint64_t* out, int count,
                          cudaStream_t st) {
  if (count <= 0) return PNB_OK;
  Fft8Tables tb;
  int rc = fft8_tables_get(&tb);
  if (rc) return rc;
  const int smem = M8 * sizeof(double2);
  PNB_CUDA(cudaFuncSetAttribute(fft8k_mul_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem));
  fft8k_mul_kernel<<<count, T8, smem, st>>>(a, b, out, tb);
  PNB_CHECK_LAUNCH("fft8k_mul_kernel");
  return PNB_OK;
}

// ---- blind rotation ----------------------------------------------------------------------------
template <bool W48>
struct Br8Layout {
  static constexpr int BUF = M8 * sizeof(double2);                // 64 KB transpose buffer
  static constexpr int ACC = 2 * M8 * sizeof(uint2);              // 64 KB: bits 32..63, pairs
  static constexpr int LO = W48 ? 2 * M8 * sizeof(ushort2) : 0;   // 32 KB: bits 16..31
  static constexpr int STAGE = 2 * 4 * T8 * sizeof(double2);      // 32 KB: 4 spectral registers
  static constexpr int STAGES = W48 ? 2 : 3;                      //   of both output polynomials
  static constexpr int ABAR = BR8_MAXN * sizeof(uint16_t);
  static constexpr int OFF_ACC = BUF;
  static constexpr int OFF_LO = OFF_ACC + ACC;
  static constexpr int OFF_RING = OFF_LO + LO;
  static constexpr int OFF_ABAR = OFF_RING + STAGES * STAGE;
  static constexpr int OFF_BAR = OFF_ABAR + ABAR;  // full[3], empty[3], abort flag, TMEM base
  static constexpr int BYTES = OFF_BAR + 64;
  // per warp 128: tw1 and tw2 factors; the 32-bit form adds 128 for the two output spectra
  static constexpr int TMEM_COLS = W48 ? 256 : 512;
};
static_assert(Br8Layout<false>::BYTES <= 227 * 1024 && Br8Layout<true>::BYTES <= 227 * 1024,
              "the N = 8192 rotation's shared layout exceeds 227 KB");

constexpr uint32_t BR8_WAIT_LIMIT = 1u << 24;

// The 48-bit form: w = v 2^-16; round(w) mod 2^48 in the top 48 bits of a torus word (pbs.cu's
// construction with 2^48 in place of 2^32).
__device__ __forceinline__ uint64_t top48_of(double w) {
  const double magic = 6755399441055744.0;
  const double magic_hi = 6755399441055744.0 * 281474976710657.0;
  const double u = fma(w, 0x1p-48, magic);
  const double q = fma(u, -281474976710656.0, magic_hi);
  return (uint64_t)__double_as_longlong(w + q) << 16;
}

// w = v 2^-32 for an exact product coefficient v: round(w) mod 2^32 with three FP64 operations
// (the construction of pbs.cu's rotation: C = 1.5 * 2^52, u = RN(w 2^-32 + C),
// q = C (1 + 2^32) - 2^32 u, and the low word of w + q).
__device__ __forceinline__ uint32_t top32_of(double w) {
  const double magic = 6755399441055744.0;
  const double magic_hi = 6755399441055744.0 * 4294967297.0;
  const double u = fma(w, 0x1p-32, magic);
  const double q = fma(u, -4294967296.0, magic_hi);
  return (uint32_t)__double2loint(w + q);
}

// L gadget levels of base 2^BETA.  With BETA * L <= 30 the accumulator keeps the top 32 bits of
// each coefficient and the digits come from the rounded top word (ties to even: with no bits
// below the word, exact ties are common, and rounding them all one way would bias every
// coefficient); otherwise it keeps the top 48 bits (a 32-bit and a 16-bit word) and the digits
// come from the 64-bit value, whose dropped low bits sit far below the product's own error.
template <int L, int BETA>
__global__ void __launch_bounds__(T8, 1) blind_rotate8k_kernel(
    const uint64_t* __restrict__ small_ct, const uint64_t* __restrict__ tvs,
    const int32_t* __restrict__ tv_idx, int tv_period, int tv_first,
    const double2* __restrict__ fbsk, uint64_t* __restrict__ out, int out_ld, int count, int n,
    Fft8Tables tb) {
  constexpr bool W48 = BETA * L > 30;
  static_assert(BETA * L <= 46, "the 48-bit accumulator holds the digits and a rounding bit");
  using Y = Br8Layout<W48>;
  constexpr int S = Y::STAGES;
  extern __shared__ __align__(128) unsigned char b8_raw[];
  double2* buf = reinterpret_cast<double2*>(b8_raw);
  uint2* acc = reinterpret_cast<uint2*>(b8_raw + Y::OFF_ACC);  // [poly][pair j]
  ushort2* lo = reinterpret_cast<ushort2*>(b8_raw + Y::OFF_LO); // [poly][pair j], 48-bit form
  const double2* ring = reinterpret_cast<const double2*>(b8_raw + Y::OFF_RING);
  uint16_t* abar = reinterpret_cast<uint16_t*>(b8_raw + Y::OFF_ABAR);
  const uint32_t full0 = tc::smem_u32(b8_raw + Y::OFF_BAR);  // full[s] at +8 s
  const uint32_t empty0 = full0 + 24;                         // empty[s] at +24 + 8 s
  volatile int* abort_s = reinterpret_cast<volatile int*>(b8_raw + Y::OFF_BAR + 48);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(b8_raw + Y::OFF_BAR + 52);
  const uint32_t ring_u32 = tc::smem_u32(b8_raw + Y::OFF_RING);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int ct = blockIdx.x;
  if (ct >= count) return;
  constexpr int LG = 14;  // log2(2N)

  // The key streams in chunks g = (i (2L) + row) 4 + c: spectral registers 4c..4c+3 of both
  // output polynomials of GGSW i, row `row` (two contiguous 16 KB pieces), into stage g mod S.
  const int total = n * (2 * L) * 4;  // <= 2^15 chunks
  auto issue = [&](int g) {
    const int st = g % S;
    const double2* f = fbsk + (size_t)(g >> 2) * 2 * M8 + (size_t)(g & 3) * 4 * T8;
    const uint32_t dst = ring_u32 + (uint32_t)st * Y::STAGE;
    tc::mbar_expect_tx(full0 + 8u * st, Y::STAGE);
#pragma unroll
    for (int h = 0; h < 2; ++h)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(dst + (uint32_t)h * (Y::STAGE / 2)), "l"(f + (size_t)h * M8),
          "r"(Y::STAGE / 2), "r"(full0 + 8u * st)
          : "memory");
  };
  if (t == 0) {
    for (int st = 0; st < S; ++st) {
      tc::mbar_init(full0 + 8u * st, 1);
      tc::mbar_init(empty0 + 8u * st, T8 / 32);
    }
    tc::fence_mbar_init();
    *abort_s = 0;
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_u32(tmem_holder), Y::TMEM_COLS);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (t == 0)
    for (int g = 0; g < S && g < total; ++g) issue(g);
  int issued = total < S ? total : S;  // thread 0's count
  // this warp's twiddle factors: lane quarter warp & 3, columns 128 (warp >> 2) + [0, 128)
  const uint32_t t_tw1 = *reinterpret_cast<volatile uint32_t*>(tmem_holder) +
                         ((uint32_t)(32 * (warp & 3)) << 16) + 128u * (uint32_t)(warp >> 2);
  const uint32_t t_tw2 = t_tw1 + 64u;
  // The 32-bit form keeps the two output spectra in tensor memory instead of registers (128
  // registers freed: no spills, 6% faster single-level; the 48-bit form, whose digit formation
  // needs the registers, keeps them in registers): chunk c (spectral registers 4c..4c+3) at
  // columns 32 c, output 0 in the first 16 columns, output 1 in the next 16.
  constexpr bool TACC = !W48;
  const uint32_t t_acc = t_tw1 + 256u;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t a[16], b[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tw_words(tb.tw1[(4 * g + q) * T8 + t], a + 4 * q);
      tw_words(tb.tw2[(4 * g + q) * 16 + (t & 15)], b + 4 * q);
    }
    tc::tmem_st_32x32_x16(t_tw1 + 16u * g, a);
    tc::tmem_st_32x32_x16(t_tw2 + 16u * g, b);
  }
  tc::tmem_st_wait();
  const uint64_t* in = small_ct + (size_t)ct * (n + 1);
  const uint64_t* tv =
      tv_idx ? tvs + (size_t)tv_idx[(int)(((long long)tv_first + ct) % tv_period)] * N8 : tvs;
  for (int i = t; i < n; i += T8) abar[i] = (uint16_t)modswitch(in[i], LG);
  const int bt = modswitch(in[n], LG);
  const int r0 = (2 * N8 - bt) & (2 * N8 - 1);
  // acc <- X^(-b) * tv on the body, zero mask; top 32 bits, rounded
  for (int j = t; j < M8; j += T8) {
    auto top = [&](int e) {
      int s = e - r0;
      bool neg = false;
      if (s < 0) { s += N8; neg = true; }
      if (s < 0) { s += N8; neg = false; }
      const uint64_t v = neg ? (uint64_t)0 - tv[s] : tv[s];
      return W48 ? v + 0x8000ull : v + 0x80000000ull;  // rounded to the kept bits
    };
    const uint64_t b0 = top(j), b1 = top(j + M8);
    acc[j] = make_uint2(0u, 0u);
    acc[M8 + j] = make_uint2((uint32_t)(b0 >> 32), (uint32_t)(b1 >> 32));
    if (W48) {
      lo[j] = make_ushort2(0, 0);
      lo[M8 + j] = make_ushort2((uint16_t)(b0 >> 16), (uint16_t)(b1 >> 16));
    }
  }
  __syncthreads();

  // gadget: T = BETA L bits; vk = w + off_h + (w >> rnd_sh & 1) rounds the top T bits of the
  // 32-bit word to nearest, ties to even, and offsets every digit by 2^(BETA-1)
  constexpr int TB = BETA * L;
  constexpr int RND_SH = 32 - TB;
  uint64_t hsum = 0;
#pragma unroll
  for (int j = 0; j < L; ++j) hsum |= (1ull << (BETA - 1)) << (BETA * j);
  const uint64_t vk_off = (1ull << (63 - TB)) + (hsum << (64 - TB));
  const uint32_t off_h = (uint32_t)(vk_off >> 32) - 1u;
  const uint32_t dmask = (1u << BETA) - 1u;
  const int dhalf = 1 << (BETA - 1);
  const int v = t;  // spectral index of this thread: k1 = v >> 4, k3 = v & 15

  for (int i = 0; i < n; ++i) {
    const int a = abar[i];
    const int ar = a & (N8 - 1);
    const uint32_t flip0 = (a >= N8) ? 0xffffffffu : 0u;
    double2 o0[16], o1[16];
    if constexpr (!TACC) {
#pragma unroll
      for (int q = 0; q < 16; ++q) o0[q] = o1[q] = make_double2(0.0, 0.0);
    }
#pragma unroll 1
    for (int row = 0; row < 2 * L; ++row) {
      const int p = row / L, lev = row % L;  // digit polynomial p (mask, body), gadget level
      const uint2* ap = acc + p * M8;
      const ushort2* lp = lo + p * M8;
      double2 x[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int j = t + T8 * m;
        const int tr = j - ar;
        const uint2 g = ap[tr & (M8 - 1)], own = ap[j];
        const bool sw = (unsigned)(tr + M8) < (unsigned)M8;
        int d0, d1;
        if constexpr (!W48) {
          const int sh = 32 - BETA * (lev + 1);
          const uint32_t w0 = (tr < 0) ? ~flip0 : flip0, w1 = (tr < -M8) ? ~flip0 : flip0;
          const uint32_t g0 = sw ? g.y : g.x, g1 = sw ? g.x : g.y;
          const uint32_t v0 = ((g0 ^ w0) - w0) - own.x;
          const uint32_t v1 = ((g1 ^ w1) - w1) - own.y;
          const uint32_t k0 = v0 + off_h + ((v0 >> RND_SH) & 1u);
          const uint32_t k1v = v1 + off_h + ((v1 >> RND_SH) & 1u);
          d0 = (int)((k0 >> sh) & dmask) - dhalf;
          d1 = (int)((k1v >> sh) & dmask) - dhalf;
        } else {
          const int sh = 64 - BETA * (lev + 1);
          const ushort2 gl = lp[tr & (M8 - 1)], ol = lp[j];
          const uint64_t f64 = flip0 ? ~0ull : 0ull;
          const uint64_t n0 = (tr < 0 ? ~0ull : 0ull) ^ f64, n1 = (tr < -M8 ? ~0ull : 0ull) ^ f64;
          const uint64_t ga = ((uint64_t)g.x << 32) | ((uint64_t)gl.x << 16);
          const uint64_t gb = ((uint64_t)g.y << 32) | ((uint64_t)gl.y << 16);
          const uint64_t g0 = sw ? gb : ga, g1 = sw ? ga : gb;
          const uint64_t v0 = ((g0 ^ n0) - n0) -
                              (((uint64_t)own.x << 32) | ((uint64_t)ol.x << 16)) + vk_off;
          const uint64_t v1 = ((g1 ^ n1) - n1) -
                              (((uint64_t)own.y << 32) | ((uint64_t)ol.y << 16)) + vk_off;
          d0 = (int)((v0 >> sh) & dmask) - dhalf;
          d1 = (int)((v1 >> sh) & dmask) - dhalf;
        }
        x[m] = make_double2((double)d0, (double)d1);
      }
      fwd8k_tm(x, buf, tb, t_tw1, t_tw2);
      // GGSW i, row (p, lev): its two output polynomials in the spectral distribution, four
      // registers per ring stage
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int g = (i * (2 * L) + row) * 4 + c;
        const int st = g % S;
        const uint32_t ph = (uint32_t)((g / S) & 1);
        if (!*abort_s && !tc::mbar_wait(full0 + 8u * st, ph, BR8_WAIT_LIMIT)) {
          *abort_s = 1;
          atomicExch(&g_br8_status, 1);
        }
        const double2* f = ring + (size_t)st * (Y::STAGE / sizeof(double2));
        if constexpr (TACC) {
          uint32_t w[32];
          if (row > 0) {
            tc::tmem_ld_32x32_nowait(t_acc + 32u * c, w);
            tc::tmem_ld_wait();
          }
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int q = 4 * c + q4;
            const double2 f0 = f[q4 * T8 + v], f1 = f[4 * T8 + q4 * T8 + v];
            const double2 s0 = row > 0 ? spec_of_words(w + 4 * q4) : make_double2(0.0, 0.0);
            const double2 s1 = row > 0 ? spec_of_words(w + 16 + 4 * q4) : make_double2(0.0, 0.0);
            const double2 xv = x[q];
            tw_words(make_double2(fma(xv.x, f0.x, fma(-xv.y, f0.y, s0.x)),
                                  fma(xv.x, f0.y, fma(xv.y, f0.x, s0.y))), w + 4 * q4);
            tw_words(make_double2(fma(xv.x, f1.x, fma(-xv.y, f1.y, s1.x)),
                                  fma(xv.x, f1.y, fma(xv.y, f1.x, s1.y))), w + 16 + 4 * q4);
          }
          tc::tmem_st_32x32(t_acc + 32u * c, w);
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int q = 4 * c + q4;
            const double2 f0 = f[q4 * T8 + v], f1 = f[4 * T8 + q4 * T8 + v];
            // o += x f as two fused multiply-adds per component
            const double2 xv = x[q];
            o0[q] = make_double2(fma(xv.x, f0.x, fma(-xv.y, f0.y, o0[q].x)),
                                 fma(xv.x, f0.y, fma(xv.y, f0.x, o0[q].y)));
            o1[q] = make_double2(fma(xv.x, f1.x, fma(-xv.y, f1.y, o1[q].x)),
                                 fma(xv.x, f1.y, fma(xv.y, f1.x, o1[q].y)));
          }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty0 + 8u * st);
        // stage st is free once every warp has read it: refill it S chunks ahead
        if (t == 0 && g + S < total && !*abort_s) {
          if (!tc::mbar_wait(empty0 + 8u * st, ph, BR8_WAIT_LIMIT)) {
            *abort_s = 1;
            atomicExch(&g_br8_status, 1);
          } else {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(g + S);
            ++issued;
          }
        }
      }
      if constexpr (TACC) tc::tmem_st_wait();  // the sums land before the next reads
    }
    // both output polynomials back to coefficients; every thread has read the accumulator
    // (the last digit pass ended on a barrier inside fwd8k) before it is updated
#pragma unroll 1
    for (int p = 0; p < 2; ++p) {
      double2 x[16];
      if constexpr (TACC) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[16];
          tc::tmem_ld_32x32_x16(t_acc + 32u * c + 16u * p, w);
          tc::tmem_ld_wait();
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) x[4 * c + q4] = spec_of_words(w + 4 * q4);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) x[q] = p == 0 ? o0[q] : o1[q];
      }
      inv8k_tm(x, buf, tb, t_tw1, t_tw2, W48 ? 0x1p-16 : 0x1p-32);
      uint2* ap = acc + p * M8;
      ushort2* lp = lo + p * M8;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int j = t + T8 * m;
        uint2 w = ap[j];
        if (!W48) {
          w.x += top32_of(x[m].x);
          w.y += top32_of(x[m].y);
        } else {
          const ushort2 l = lp[j];
          const uint64_t a0 = (((uint64_t)w.x << 32) | ((uint64_t)l.x << 16)) + top48_of(x[m].x);
          const uint64_t a1 = (((uint64_t)w.y << 32) | ((uint64_t)l.y << 16)) + top48_of(x[m].y);
          w = make_uint2((uint32_t)(a0 >> 32), (uint32_t)(a1 >> 32));
          lp[j] = make_ushort2((uint16_t)(a0 >> 16), (uint16_t)(a1 >> 16));
        }
        ap[j] = w;
      }
    }
    __syncthreads();
    if (*abort_s) break;  // uniform: every thread reads the flag after the same barrier
  }
  // the copies still in flight (only after a wait gave up) land before the block exits
  if (t == 0 && *abort_s)
    for (int g = issued - S < 0 ? 0 : issued - S; g < issued; ++g)
      (void)tc::mbar_wait(full0 + 8u * (uint32_t)(g % S), (uint32_t)((g / S) & 1),
                          BR8_WAIT_LIMIT);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(*reinterpret_cast<volatile uint32_t*>(tmem_holder), Y::TMEM_COLS);
  }
  if (*abort_s) return;
  // sample extraction of coefficient 0 under the big key
  uint64_t* o = out + (size_t)ct * out_ld;
  auto coef = [&](int p, int e) {
    const uint2 w = acc[p * M8 + (e & (M8 - 1))];
    uint64_t v = (uint64_t)(e < M8 ? w.x : w.y) << 32;
    if (W48) {
      const ushort2 l = lo[p * M8 + (e & (M8 - 1))];
      v |= (uint64_t)(e < M8 ? l.x : l.y) << 16;
    }
    return v;
  };
  for (int e = t; e < N8; e += T8) o[e] = (e == 0) ? coef(0, 0) : (uint64_t)0 - coef(0, N8 - e);
  if (t == 0) o[N8] = coef(1, 0);
}

template <int L, int BETA>
static int launch8k(const pnb_keys* K, const uint64_t* tvs, const int32_t* tv_idx, int period,
                    int first, const uint64_t* small, uint64_t* out, int out_ld, int count,
                    cudaStream_t st) {
  Fft8Tables tb;
  int rc = fft8_tables_get(&tb);
  if (rc) return rc;
  constexpr int smem = Br8Layout<(BETA * L > 30)>::BYTES;
  PNB_CUDA(cudaFuncSetAttribute(blind_rotate8k_kernel<L, BETA>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  blind_rotate8k_kernel<L, BETA><<<count, T8, smem, st>>>(small, tvs, tv_idx, period, first,
                                                          K->fbsk, out, out_ld, count, K->p.n,
                                                          tb);
  PNB_CHECK_LAUNCH("blind_rotate8k_kernel");
  return PNB_OK;
}

bool br8k_supported(const pnb_params& p) {
  return p.k == 1 && p.N == N8 && p.n > 0 && p.n <= BR8_MAXN &&
         ((p.pbs_level == 1 && p.pbs_base_log == 23) ||
          (p.pbs_level == 2 && p.pbs_base_log == 15) ||
          (p.pbs_level == 4 && p.pbs_base_log == 11));
}

int blind_rotate_8k(const pnb_keys* K, const uint64_t* tvs, const int32_t* tv_idx, int period,
                    int first, const uint64_t* small, uint64_t* out, int out_ld, int count,
                    cudaStream_t st) {
  if (!br8k_supported(K->p)) {
    set_error("blind rotation at N = 8192: compiled for k = 1, n <= %d and the gadgets "
              "(2^23, 1), (2^15, 2), (2^11, 4) (got n=%d base_log=%d level=%d)", BR8_MAXN, K->p.n,
              K->p.pbs_base_log, K->p.pbs_level);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count <= 0) return PNB_OK;
  if (K->p.pbs_level == 1)
    return launch8k<1, 23>(K, tvs, tv_idx, period, first, small, out, out_ld, count, st);
  if (K->p.pbs_level == 2)
    return launch8k<2, 15>(K, tvs, tv_idx, period, first, small, out, out_ld, count, st);
  return launch8k<4, 11>(K, tvs, tv_idx, period, first, small, out, out_ld, count, st);
}

}  // namespace pnb
