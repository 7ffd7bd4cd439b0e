// pbs.cu -- batched programmable bootstrapping on B200: keyswitch, blind rotation over the
// Fourier bootstrapping key, fused sample extraction; Fourier conversion of the key.
//
// Restates what tfhe 1.6.3's shortint ServerKey::apply_lookup_table runs per ciphertext for
// the KS_PBS order (reference call sites runtime/src/ops/activation.rs:115,
// runtime/src/ops/requant.rs:232), batched over every ciphertext of a layer:
//   1. keyswitch big key (k*N) -> small key (n), signed gadget digits (ks_base_log, ks_level);
//   2. modulus switch of the small ciphertext to Z_{2N};
//   3. blind rotation ACC <- ACC + ExtProd(BSK_i, X^{a_i} ACC - ACC) for i < n, the external
//      product evaluated through the f64 negacyclic FFT (fft1024.cuh);
//   4. sample extraction of coefficient 0 (fused into the blind rotation's epilogue).
#include <cmath>
#include <cstdio>
#include <mutex>
#include <vector>

#include "fft1024.cuh"
#include "pnb_internal.cuh"
#include "pnb_keys.h"

namespace pnb {

// ------------------------------------------------------------------------------------------
// FFT tables (one set per device, built on first use).
// ------------------------------------------------------------------------------------------
static std::mutex g_tab_mu;
static FftTables g_tab[64];
static bool g_tab_ok[64];

static int bitrev5(int v) {
  int r = 0;
  for (int b = 0; b < 5; ++b)
    if (v & (1 << b)) r |= 1 << (4 - b);
  return r;
}

int fft_tables_get(FftTables* out) {
  int dev = 0;
  PNB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("device index %d out of range", dev);
    return PNB_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_tab_mu);
  if (!g_tab_ok[dev]) {
    const int N = FFT_N, M = FFT_M;
    const long double PI = 3.141592653589793238462643383279502884L;
    std::vector<double2> wf(M), wi(M), twf(32), twi(32);
    auto expi = [&](long double ang) {
      return make_double2((double)cosl(ang), (double)sinl(ang));
    };
    for (int r = 0; r < 32; ++r)
      for (int l = 0; l < 32; ++l) {
        // zeta^l W^{l k2}, k2 = bitrev(r): angle pi l / N - 2 pi (l k2 mod M) / M
        long long e = ((long long)l * bitrev5(r)) % M;
        wf[r * 32 + l] = expi(PI * l / N - 2.0L * PI * e / M);
      }
    for (int n = 0; n < 32; ++n)
      for (int l = 0; l < 32; ++l) {
        // zeta^{-n} W^{-n k2}, k2 = bitrev(l)
        long long e = ((long long)n * bitrev5(l)) % M;
        wi[n * 32 + l] = expi(-PI * n / N + 2.0L * PI * e / M);
      }
    for (int m = 0; m < 32; ++m) {
      twf[m] = expi(PI * (32.0L * m) / N);
      double2 t = expi(-PI * (32.0L * m) / N);
      twi[m] = make_double2(t.x / M, t.y / M);
    }
    FftTables t{};
    PNB_CUDA(cudaMalloc(&t.wf, sizeof(double2) * M));
    PNB_CUDA(cudaMalloc(&t.wi, sizeof(double2) * M));
    PNB_CUDA(cudaMalloc(&t.twf, sizeof(double2) * 32));
    PNB_CUDA(cudaMalloc(&t.twi, sizeof(double2) * 32));
    PNB_CUDA(cudaMemcpy(t.wf, wf.data(), sizeof(double2) * M, cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.wi, wi.data(), sizeof(double2) * M, cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.twf, twf.data(), sizeof(double2) * 32, cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.twi, twi.data(), sizeof(double2) * 32, cudaMemcpyHostToDevice));
    g_tab[dev] = t;
    g_tab_ok[dev] = true;
  }
  *out = g_tab[dev];
  return PNB_OK;
}

// Coefficient t of X^r * P (negacyclic), r in [0, 2N).
__device__ __forceinline__ uint64_t rot_coef(const uint64_t* P, int t, int r) {
  int s = t - r;
  bool neg = false;
  if (s < 0) { s += FFT_N; neg = true; }
  if (s < 0) { s += FFT_N; neg = false; }
  uint64_t v = P[s];
  return neg ? (uint64_t)0 - v : v;
}

// ------------------------------------------------------------------------------------------
// Fourier conversion of the bootstrapping key: one warp per polynomial.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) bsk_to_fourier_kernel(const uint64_t* __restrict__ bsk,
                                                             double2* __restrict__ fbsk,
                                                             int polys, FftTables tb) {
  extern __shared__ double2 fsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int poly = blockIdx.x * 4 + warp;
  if (poly >= polys) return;
  const uint64_t* a = bsk + (size_t)poly * FFT_N;
  double2 x[FFT_R];
#pragma unroll
  for (int m = 0; m < 32; ++m) {
    const int j = lane + 32 * m;
    x[m] = make_double2(__ll2double_rn((long long)a[j]), __ll2double_rn((long long)a[j + FFT_M]));
  }
  fft_forward(x, fsm + warp * FFT_M, lane, tb);
  double2* o = fbsk + (size_t)poly * FFT_M;
#pragma unroll
  for (int r = 0; r < 32; ++r) o[r * 32 + lane] = x[r];
}

int bsk_to_fourier(const uint64_t* bsk_dev, double2* fbsk_dev, int polys, cudaStream_t st) {
  FftTables tb;
  int rc = fft_tables_get(&tb);
  if (rc) return rc;
  const int smem = 4 * FFT_M * sizeof(double2);
  PNB_CUDA(cudaFuncSetAttribute(bsk_to_fourier_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  bsk_to_fourier_kernel<<<(polys + 3) / 4, 128, smem, st>>>(bsk_dev, fbsk_dev, polys, tb);
  PNB_CHECK_LAUNCH("bsk_to_fourier_kernel");
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// Keyswitch: out[c][t] = (t == n ? b_c : 0) - sum_{i,j} digit_{c,i,j} * KSK[i][j][t].
// Block = 128 threads covering 256 output columns for KS_CT ciphertexts.
// ------------------------------------------------------------------------------------------
constexpr int KS_CT = 32;    // ciphertexts per block
constexpr int KS_ICH = 16;   // input coefficients staged per round
constexpr int KS_MAXL = 8;   // maximum keyswitch levels

__global__ void __launch_bounds__(128) keyswitch_kernel(const uint64_t* __restrict__ in,
                                                        uint64_t* __restrict__ out,
                                                        const uint64_t* __restrict__ ksk,
                                                        int count, int n, int big, int base_log,
                                                        int level) {
  __shared__ int8_t dig[KS_CT][KS_ICH * KS_MAXL];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * 256 + tid, t1 = t0 + 128;
  const int c0 = blockIdx.y * KS_CT;
  const int nct = min(KS_CT, count - c0);
  const int row = n + 1;
  uint64_t acc0[KS_CT], acc1[KS_CT];
#pragma unroll
  for (int c = 0; c < KS_CT; ++c) { acc0[c] = 0; acc1[c] = 0; }
  const bool ok0 = t0 < row, ok1 = t1 < row;
  const int total = base_log * level;
  const uint64_t mask = (1ull << base_log) - 1, half = 1ull << (base_log - 1);

  for (int i0 = 0; i0 < big; i0 += KS_ICH) {
    __syncthreads();
    for (int e = tid; e < KS_CT * KS_ICH; e += 128) {
      const int c = e / KS_ICH, ii = e % KS_ICH;
      if (c < nct && i0 + ii < big) {
        uint64_t a = in[(size_t)(c0 + c) * (big + 1) + i0 + ii];
        uint64_t st = (a >> (64 - total)) + ((a >> (63 - total)) & 1u);
        for (int j = level - 1; j >= 0; --j) {
          uint64_t d = st & mask;
          st >>= base_log;
          bool neg = d >= half;
          dig[c][ii * KS_MAXL + j] = (int8_t)(neg ? (int64_t)d - (int64_t)(1ull << base_log)
                                                  : (int64_t)d);
          st += neg ? 1u : 0u;
        }
      } else {
        for (int j = 0; j < level; ++j) dig[c][ii * KS_MAXL + j] = 0;
      }
    }
    __syncthreads();
    const int iimax = min(KS_ICH, big - i0);
    for (int ii = 0; ii < iimax; ++ii) {
      for (int j = 0; j < level; ++j) {
        const uint64_t* kr = ksk + ((size_t)(i0 + ii) * level + j) * row;
        const uint64_t k0 = ok0 ? __ldg(kr + t0) : 0, k1 = ok1 ? __ldg(kr + t1) : 0;
#pragma unroll
        for (int c = 0; c < KS_CT; ++c) {
          const uint64_t d = (uint64_t)(int64_t)dig[c][ii * KS_MAXL + j];
          acc0[c] -= d * k0;
          acc1[c] -= d * k1;
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < KS_CT; ++c) {
    if (c < nct) {
      const uint64_t b = in[(size_t)(c0 + c) * (big + 1) + big];
      if (ok0) out[(size_t)(c0 + c) * row + t0] = acc0[c] + (t0 == n ? b : 0);
      if (ok1) out[(size_t)(c0 + c) * row + t1] = acc1[c] + (t1 == n ? b : 0);
    }
  }
}

int keyswitch_launch(const pnb_keys* K, const uint64_t* in, uint64_t* out, int count,
                     cudaStream_t st) {
  const pnb_params& p = K->p;
  // digits are staged as int8: |digit| <= 2^(base_log-1) must fit
  if (p.ks_level > KS_MAXL || p.ks_base_log * p.ks_level >= 64 || p.ks_base_log < 1 ||
      p.ks_base_log > 7) {
    set_error("keyswitch: unsupported ks_base_log=%d ks_level=%d", p.ks_base_log, p.ks_level);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count <= 0) return PNB_OK;
  dim3 grid((p.n + 1 + 255) / 256, (count + KS_CT - 1) / KS_CT);
  keyswitch_kernel<<<grid, 128, 0, st>>>(in, out, K->ksk, count, p.n, p.k * p.N, p.ks_base_log,
                                         p.ks_level);
  PNB_CHECK_LAUNCH("keyswitch_kernel");
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// Blind rotation + sample extraction, k = 1, pbs_level = 1, N = 2048.
// One block of 2 warps per ciphertext; warp p owns GLWE polynomial p (0 = mask, 1 = body).
// ------------------------------------------------------------------------------------------
constexpr int BR_MAXN = 1024;  // maximum small LWE dimension supported by the smem layout

struct BrSmem {
  uint64_t acc[2][FFT_N];
  double2 buf[2][FFT_M];
  uint16_t abar[BR_MAXN];
};

__global__ void __launch_bounds__(64) blind_rotate_k1l1_kernel(
    const uint64_t* __restrict__ small_ct, const uint64_t* __restrict__ tv,
    const double2* __restrict__ fbsk, uint64_t* __restrict__ out, int n, int base_log,
    FftTables tb) {
  extern __shared__ __align__(16) unsigned char br_raw[];
  BrSmem& S = *reinterpret_cast<BrSmem*>(br_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ct = blockIdx.x;
  const uint64_t* in = small_ct + (size_t)ct * (n + 1);
  constexpr int LG = 12;  // log2(2N)
  for (int i = threadIdx.x; i < n; i += 64) S.abar[i] = (uint16_t)modswitch(in[i], LG);
  const int bt = modswitch(in[n], LG);
  const int r0 = (2 * FFT_N - bt) & (2 * FFT_N - 1);
  for (int t = threadIdx.x; t < FFT_N; t += 64) {
    S.acc[0][t] = 0;
    S.acc[1][t] = rot_coef(tv, t, r0);
  }
  __syncthreads();

  uint64_t* my = S.acc[warp];
  double2* mybuf = S.buf[warp];
  const double2* otherbuf = S.buf[warp ^ 1];
  const uint64_t rnd = 1ull << (63 - base_log);
  const uint64_t dmask = (1ull << base_log) - 1, dhalf = 1ull << (base_log - 1);

  for (int i = 0; i < n; ++i) {
    const int a = S.abar[i];
    if (a == 0) continue;
    double2 x[FFT_R];
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      // Keep the shared-memory loads of a few coefficients in flight at a time: hoisting all
      // 64 of them ahead of the conversions would exceed the register budget.
      if ((m & 7) == 0) asm volatile("" ::: "memory");
      const int j = lane + 32 * m;
      const uint64_t v0 = rot_coef(my, j, a) - my[j];
      const uint64_t v1 = rot_coef(my, j + FFT_M, a) - my[j + FFT_M];
      // single-level signed digit: round to base_log bits, centre in [-B/2, B/2)
      uint64_t s0 = ((v0 + rnd) >> (64 - base_log)) & dmask;
      uint64_t s1 = ((v1 + rnd) >> (64 - base_log)) & dmask;
      const int64_t d0 = s0 >= dhalf ? (int64_t)s0 - (int64_t)(dmask + 1) : (int64_t)s0;
      const int64_t d1 = s1 >= dhalf ? (int64_t)s1 - (int64_t)(dmask + 1) : (int64_t)s1;
      x[m] = make_double2(small_int_to_f64(d0), small_int_to_f64(d1));
    }
    fft_forward(x, mybuf, lane, tb);
#pragma unroll
    for (int r = 0; r < 32; ++r) mybuf[r * 32 + lane] = x[r];
    __syncthreads();
    // Output polynomial c = warp: D_own * F[own row][c] + D_other * F[other row][c].
    const double2* g = fbsk + (size_t)i * 4 * FFT_M;
    const double2* f_own = g + (size_t)(warp * 2 + warp) * FFT_M;
    const double2* f_oth = g + (size_t)((warp ^ 1) * 2 + warp) * FFT_M;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      if ((r & 3) == 0) asm volatile("" ::: "memory");
      const int e = r * 32 + lane;
      const double2 fo = __ldg(&f_own[e]), ft = __ldg(&f_oth[e]);
      const double2 dt = otherbuf[e];
      const double2 p0 = cmul(x[r], fo);
      x[r] = make_double2(p0.x + fma(dt.x, ft.x, -dt.y * ft.y),
                          p0.y + fma(dt.x, ft.y, dt.y * ft.x));
    }
    __syncthreads();
    fft_inverse(x, mybuf, lane, tb);
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if ((m & 7) == 0) asm volatile("" ::: "memory");
      const int j = lane + 32 * m;
      my[j] += f64_to_torus(x[m].x);
      my[j + FFT_M] += f64_to_torus(x[m].y);
    }
    __syncwarp();
  }
  __syncthreads();
  // Sample extraction of coefficient 0 into an LWE of dimension N under the big key.
  uint64_t* o = out + (size_t)ct * (FFT_N + 1);
  for (int t = threadIdx.x; t < FFT_N; t += 64)
    o[t] = (t == 0) ? S.acc[0][0] : (uint64_t)0 - S.acc[0][FFT_N - t];
  if (threadIdx.x == 0) o[FFT_N] = S.acc[1][0];
}

static bool br_supported(const pnb_params& p) {
  return p.k == 1 && p.N == FFT_N && p.pbs_level == 1 && p.n <= BR_MAXN && p.n > 0 &&
         p.pbs_base_log >= 2 && p.pbs_base_log <= 40;
}

int blind_rotate_launch(const pnb_keys* K, const uint64_t* tv, const uint64_t* small,
                        uint64_t* out, int count, cudaStream_t st) {
  if (!br_supported(K->p)) {
    set_error("blind rotation: compiled kernels cover k=1, N=2048, pbs_level=1, n<=%d (got "
              "k=%d N=%d level=%d n=%d)", BR_MAXN, K->p.k, K->p.N, K->p.pbs_level, K->p.n);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count <= 0) return PNB_OK;
  FftTables tb;
  int rc = fft_tables_get(&tb);
  if (rc) return rc;
  const int smem = sizeof(BrSmem);
  PNB_CUDA(cudaFuncSetAttribute(blind_rotate_k1l1_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  blind_rotate_k1l1_kernel<<<count, 64, smem, st>>>(small, tv, K->fbsk, out, K->p.n,
                                                    K->p.pbs_base_log, tb);
  PNB_CHECK_LAUNCH("blind_rotate_k1l1_kernel");
  return PNB_OK;
}

size_t pbs_workspace_bytes(const pnb_keys* K, int count) {
  if (!K || count <= 0) return 0;
  return (size_t)count * (K->p.n + 1) * sizeof(uint64_t);
}

int pbs_batch(const pnb_keys* K, const uint64_t* tv, const uint64_t* in, uint64_t* out,
              int count, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!br_supported(K->p)) {
    set_error("pbs: compiled kernels cover k=1, N=2048, pbs_level=1, n<=%d (got k=%d N=%d "
              "level=%d n=%d)", BR_MAXN, K->p.k, K->p.N, K->p.pbs_level, K->p.n);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count == 0) return PNB_OK;
  int rc = PNB_OK;
  const size_t need = pbs_workspace_bytes(K, count);
  uint64_t* small = nullptr;
  bool own = false;
  if (ws) {
    if (ws_bytes < need) {
      set_error("pbs: workspace of %zu bytes is smaller than the %zu bytes needed", ws_bytes,
                need);
      return PNB_ERR_INVALID;
    }
    small = static_cast<uint64_t*>(ws);
  } else {
    cudaError_t e = cudaMallocAsync((void**)&small, need, st);
    if (e != cudaSuccess) return cuda_status(e, "cudaMallocAsync(pbs workspace)");
    own = true;
  }
  rc = keyswitch_launch(K, in, small, count, st);
  if (rc == PNB_OK) rc = blind_rotate_launch(K, tv, small, out, count, st);
  if (own) {
    cudaError_t e = cudaFreeAsync(small, st);
    if (rc == PNB_OK && e != cudaSuccess) rc = cuda_status(e, "cudaFreeAsync(pbs workspace)");
  }
  return rc;
}

// ------------------------------------------------------------------------------------------
// Test vector of a lookup table.
// ------------------------------------------------------------------------------------------
__global__ void test_vector_kernel(const uint64_t* __restrict__ lut, int lut_len,
                                   uint64_t delta_out, uint64_t* __restrict__ tv, int N) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  const int box = N / lut_len, half = box / 2;
  const int m = (j + half) / box;
  tv[j] = (m < lut_len) ? lut[m] * delta_out : (uint64_t)0 - lut[m - lut_len] * delta_out;
}

int test_vector(const pnb_keys* K, const uint64_t* lut_host, int lut_len, uint64_t delta_out,
                uint64_t* tv, cudaStream_t st) {
  const int N = K->p.N;
  if (lut_len <= 0 || lut_len > N || (N % lut_len) != 0) {
    set_error("test_vector: lut_len %d must divide N = %d", lut_len, N);
    return PNB_ERR_INVALID;
  }
  uint64_t* d_lut = nullptr;
  PNB_CUDA(cudaMallocAsync((void**)&d_lut, sizeof(uint64_t) * lut_len, st));
  PNB_CUDA(cudaMemcpyAsync(d_lut, lut_host, sizeof(uint64_t) * lut_len, cudaMemcpyHostToDevice,
                           st));
  test_vector_kernel<<<(N + 255) / 256, 256, 0, st>>>(d_lut, lut_len, delta_out, tv, N);
  PNB_CHECK_LAUNCH("test_vector_kernel");
  PNB_CUDA(cudaFreeAsync(d_lut, st));
  // The host LUT buffer must stay valid until the copy above completes.
  PNB_CUDA(cudaStreamSynchronize(st));
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// Diagnostic: negacyclic products through the FFT.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(32) fft_mul_kernel(const int64_t* __restrict__ a,
                                                     const uint64_t* __restrict__ b,
                                                     uint64_t* __restrict__ out, FftTables tb) {
  __shared__ double2 buf[FFT_M];
  const int lane = threadIdx.x, poly = blockIdx.x;
  const int64_t* pa = a + (size_t)poly * FFT_N;
  const uint64_t* pb = b + (size_t)poly * FFT_N;
  double2 x[FFT_R], y[FFT_R];
#pragma unroll
  for (int m = 0; m < 32; ++m) {
    const int j = lane + 32 * m;
    x[m] = make_double2(__ll2double_rn(pa[j]), __ll2double_rn(pa[j + FFT_M]));
    y[m] = make_double2(__ll2double_rn((long long)pb[j]),
                        __ll2double_rn((long long)pb[j + FFT_M]));
  }
  fft_forward(x, buf, lane, tb);
  fft_forward(y, buf, lane, tb);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], y[r]);
  fft_inverse(x, buf, lane, tb);
  uint64_t* po = out + (size_t)poly * FFT_N;
#pragma unroll
  for (int m = 0; m < 32; ++m) {
    const int j = lane + 32 * m;
    po[j] = f64_to_torus(x[m].x);
    po[j + FFT_M] = f64_to_torus(x[m].y);
  }
}

int fft_negacyclic_mul(int N, const int64_t* a, const uint64_t* b, uint64_t* out, int count,
                       cudaStream_t st) {
  if (N != FFT_N) {
    set_error("fft_negacyclic_mul: compiled for N = %d, got %d", FFT_N, N);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count <= 0) return PNB_OK;
  FftTables tb;
  int rc = fft_tables_get(&tb);
  if (rc) return rc;
  fft_mul_kernel<<<count, 32, 0, st>>>(a, b, out, tb);
  PNB_CHECK_LAUNCH("fft_mul_kernel");
  return PNB_OK;
}

}  // namespace pnb
