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
#include "tc_primitives.cuh"

namespace pnb {

// Device-side status word of the blind rotation: non-zero when its bounded wait ran out.
__device__ int g_br_status;

int br_status_read_and_clear(int* out) {
  int v = 0, v8 = 0;
  PNB_CUDA(cudaMemcpyFromSymbol(&v, g_br_status, sizeof(int)));
  const int zero = 0;
  PNB_CUDA(cudaMemcpyToSymbol(g_br_status, &zero, sizeof(int)));
  const int rc = br8_status_read_and_clear(&v8);  // the N = 8192 rotation's word
  if (rc) return rc;
  *out = v | v8;
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// FFT tables (one set per device, built on first use).
// ------------------------------------------------------------------------------------------
static std::mutex g_tab_mu;
static FftTables g_tab[64];
static bool g_tab_ok[64];

// T(r, l) = rho_r^l, rho_r = exp(i pi (1 + 4 bitrev(r)) / 2048): angle pi e / 2048 with the
// exponent e reduced mod 4096 in integers first, evaluated in long double on the host.
static double2 mid_twiddle(int r, int l);

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
    const int M = FFT_M;
    std::vector<double2> wf(M), wi(M);
    for (int r = 0; r < 32; ++r)
      for (int l = 0; l < 32; ++l) {
        wf[r * 32 + l] = mid_twiddle(r, l);
        const double2 t = mid_twiddle(l, r);
        wi[r * 32 + l] = make_double2(t.x, -t.y);
      }
    FftTables t{};
    PNB_CUDA(cudaMalloc(&t.wf, sizeof(double2) * M));
    PNB_CUDA(cudaMalloc(&t.wi, sizeof(double2) * M));
    PNB_CUDA(cudaMemcpy(t.wf, wf.data(), sizeof(double2) * M, cudaMemcpyHostToDevice));
    PNB_CUDA(cudaMemcpy(t.wi, wi.data(), sizeof(double2) * M, cudaMemcpyHostToDevice));
    g_tab[dev] = t;
    g_tab_ok[dev] = true;
  }
  *out = g_tab[dev];
  return PNB_OK;
}

static double2 mid_twiddle(int r, int l) {
  const long double PI = 3.141592653589793238462643383279502884L;
  const long long e = ((long long)l * (1 + 4 * bitrev5(r))) % 4096;
  const long double ang = PI * (long double)e / 2048.0L;
  return make_double2((double)cosl(ang), (double)sinl(ang));
}

// True when the current device's FFT tables exist (never allocates).
bool fft_tables_ready() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lk(g_tab_mu);
  return g_tab_ok[dev];
}

// Coefficient t of X^r * P (negacyclic), r in [0, 2N).
// Test-vector selection: ciphertext ct starts from tvs[idx[(first + ct) % period]]
// (idx == nullptr: every ciphertext starts from tvs).
struct TvSel {
  const uint64_t* tvs;
  const int32_t* idx;
  int period;
  int first;
};
__device__ __forceinline__ const uint64_t* tv_of(const TvSel& s, int ct) {
  return s.idx ? s.tvs + (size_t)s.idx[(int)(((long long)s.first + ct) % s.period)] * FFT_N
               : s.tvs;
}

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
// Keyswitch (tensor cores, ks_tc.cu): digit scratch from `digits` or the stream allocator.
// ------------------------------------------------------------------------------------------
int keyswitch_launch(const pnb_keys* K, const uint64_t* in, uint64_t* out, int count,
                     void* digits, cudaStream_t st, int in_ld) {
  if (count <= 0) return PNB_OK;
  void* d = digits;
  bool own = false;
  if (!d) {
    cudaError_t e = cudaMallocAsync(&d, ks_tc_workspace_bytes(K->p, count), st);
    if (e != cudaSuccess) return cuda_status(e, "cudaMallocAsync(keyswitch digits)");
    own = true;
  }
  int rc = keyswitch_tc(K, in, out, count, d, st, in_ld);
  if (own) {
    cudaError_t e = cudaFreeAsync(d, st);
    if (rc == PNB_OK && e != cudaSuccess) rc = cuda_status(e, "cudaFreeAsync(keyswitch digits)");
  }
  return rc;
}

// ------------------------------------------------------------------------------------------
// Blind rotation + sample extraction, k = 1, pbs_level = 1, N = 2048.
//
// A block bootstraps CPB ciphertexts in lockstep; warp (2c + p) owns GLWE polynomial p
// (0 = mask, 1 = body) of ciphertext c.  The accumulator lives in shared memory as the top 32
// bits of each torus coefficient: the f64 FFT product already carries ~2^37 of rounding error
// per coefficient, so the dropped low word (<= 2^32, a random walk of ~2^35 after n updates)
// sits far below both that and the bootstrap's own output noise (~2^49).  Warps of the same
// output polynomial read the same bootstrapping-key lines right after a block barrier, so the
// second and later ciphertexts of a block find them in L1.
// ------------------------------------------------------------------------------------------
constexpr int BR_MAXN = 1024;  // maximum small LWE dimension supported by the smem layout

// Where the rotation kernels' FFT constants live (1: constant bank, 0: literals); chosen per
// kernel by register pressure.
#ifndef PNB_BR_CBANK
#define PNB_BR_CBANK 1
#endif
#ifndef PNB_ML_CBANK
#define PNB_ML_CBANK 1
#endif

template <int CPB>
struct BrLayout {
  static constexpr int WARPS = 2 * CPB;
  static constexpr int SCRATCH = FFT_M * sizeof(double);            // 8 KB per warp
  static constexpr int ACC = FFT_N * sizeof(uint32_t);              // 8 KB per warp
  static constexpr int BSK = 4 * FFT_M * sizeof(double2);           // 64 KB: one GGSW (k=1,l=1)
  static constexpr int ABAR = BR_MAXN * sizeof(uint16_t);           // 2 KB per ciphertext
  static constexpr int OFF_ACC = WARPS * SCRATCH;
  static constexpr int OFF_BSK = OFF_ACC + WARPS * ACC;
  static constexpr int OFF_WF = OFF_BSK + BSK;  // 16 KB twiddles (both directions, swizzled)
  static constexpr int OFF_ABAR = OFF_WF + FFT_M * (int)sizeof(double2);
  static constexpr int OFF_BAR = OFF_ABAR + CPB * ABAR;
  static constexpr int BYTES = OFF_BAR + 16;
};

// The blind rotation's inverse FFT leaves w = v * 2^-32, v the exact product coefficient
// (|v| < 2^100).  Return round(w) mod 2^32 -- the top word of the torus value -- with three FP64
// operations and no integer work.  With C = 1.5 * 2^52: u = RN(w 2^-32 + C) = C + k,
// k = round(w / 2^32); q = C (1 + 2^32) - 2^32 u = C - 2^32 k exactly (a multiple of 2^32 below
// 2^72); w + q = (w - 2^32 k) + C with |w - 2^32 k| <= 2^31, so its rounding to the unit grid of
// [2^52, 2^53) is C + round(w - 2^32 k), whose low word is round(w) mod 2^32 (C = 0 mod 2^32).
__device__ __forceinline__ uint32_t scaled_f64_to_top32(double w) {
  const double magic = 6755399441055744.0;            // 1.5 * 2^52
  const double magic_hi = 6755399441055744.0 * 4294967297.0;  // C (1 + 2^32), exact
  const double u = fma(w, 0x1p-32, magic);
  const double q = fma(u, -4294967296.0, magic_hi);
  return (uint32_t)__double2loint(w + q);
}

// Named barrier over the two warps of one ciphertext.
__device__ __forceinline__ void pair_sync(int pair) {
  asm volatile("bar.sync %0, 64;" ::"r"(pair + 1) : "memory");
}

constexpr uint32_t BR_WAIT_LIMIT = 1u << 24;

// Stage GGSW number i of the Fourier bootstrapping key (64 KB) into shared memory.
__device__ __forceinline__ void br_stage_ggsw(uint32_t dst, const double2* src, uint32_t bar) {
  tc::mbar_expect_tx(bar, 4 * FFT_M * sizeof(double2));
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst + q * FFT_M * 16u), "l"(src + q * FFT_M), "r"(FFT_M * 16u), "r"(bar)
        : "memory");
  }
}

template <int CPB>
__global__ void __launch_bounds__(64 * CPB, 1) blind_rotate_kernel(
    const uint64_t* __restrict__ small_ct, TvSel sel,
    const double2* __restrict__ fbsk, uint64_t* __restrict__ out, int out_ld, int count, int n,
    int base_log, FftTables tb) {
  using L = BrLayout<CPB>;
  extern __shared__ __align__(128) unsigned char br_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = warp >> 1, p = warp & 1;
  const int ct = blockIdx.x * CPB + cl;
  const bool valid = ct < count;
  constexpr int LG = 12;  // log2(2N)
  double* buf = reinterpret_cast<double*>(br_raw) + warp * FFT_M;
  double2* xbuf = reinterpret_cast<double2*>(buf);  // the same 8 KB seen as 512 complex
  const double2* obuf = reinterpret_cast<const double2*>(reinterpret_cast<double*>(br_raw) +
                                                         (warp ^ 1) * FFT_M);
  // accumulator coefficients (j, j + M) side by side: acc2[j] = (acc[j], acc[j + M]), j < M
  uint2* acc2 = reinterpret_cast<uint2*>(br_raw + L::OFF_ACC) + warp * FFT_M;
  auto acc_at = [&](int e) { return e < FFT_M ? acc2[e].x : acc2[e - FFT_M].y; };
  const double2* bsk_s = reinterpret_cast<const double2*>(br_raw + L::OFF_BSK);
  double2* wf_s = reinterpret_cast<double2*>(br_raw + L::OFF_WF);
  uint16_t* abar = reinterpret_cast<uint16_t*>(br_raw + L::OFF_ABAR) + cl * BR_MAXN;
  const uint32_t bar = tc::smem_u32(br_raw + L::OFF_BAR);
  volatile int* abort_s = reinterpret_cast<volatile int*>(br_raw + L::OFF_BAR + 8);
  const uint32_t bsk_dst = tc::smem_u32(br_raw + L::OFF_BSK);

  if (threadIdx.x == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
    *abort_s = 0;
  }
  for (int e = threadIdx.x; e < FFT_M; e += 64 * CPB) wf_s[tw_swz(e >> 5, e & 31)] = tb.wf[e];
  __syncthreads();
  if (threadIdx.x == 0) br_stage_ggsw(bsk_dst, fbsk, bar);

  const uint64_t* in = small_ct + (size_t)(valid ? ct : 0) * (n + 1);
  const uint64_t* tv = tv_of(sel, valid ? ct : 0);
  const int t64 = threadIdx.x & 63;
  for (int i = t64; i < n; i += 64) abar[i] = valid ? (uint16_t)modswitch(in[i], LG) : 0;
  const int bt = valid ? modswitch(in[n], LG) : 0;
  const int r0 = (2 * FFT_N - bt) & (2 * FFT_N - 1);
  for (int t = lane; t < FFT_M; t += 32) {
    auto top = [&](int e) { return (uint32_t)((rot_coef(tv, e, r0) + 0x80000000ull) >> 32); };
    acc2[t] = (p == 0) ? make_uint2(0u, 0u) : make_uint2(top(t), top(t + FFT_M));
  }
  __syncthreads();

  const int shift = 32 - base_log;
  const uint32_t rnd = 1u << (shift - 1);
  const double2* f_own = bsk_s + (size_t)(p * 2 + p) * FFT_M;
  const double2* f_oth = bsk_s + (size_t)((p ^ 1) * 2 + p) * FFT_M;

  for (int i = 0; i < n; ++i) {
    const int a = abar[i];
    // X^a = (-1)^(a >= N) X^(a mod N): rotate by ar in [0, N), flip the sign where it wraps.
    const int ar = a & (FFT_N - 1);
    const uint32_t flip0 = (a >= FFT_N) ? 0xffffffffu : 0u;
    double2 x[FFT_R];
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if ((m & 7) == 0) asm volatile("" ::: "memory");
      const int j = lane + 32 * m;
      // Coefficients t = j - ar and t + M of X^ar acc share the pair slot t mod M: t >= 0 reads
      // (x, y) as they are, -M <= t < 0 reads (-y, x), t < -M reads (-x, -y).
      const int t = j - ar;
      const uint2 g = acc2[t & (FFT_M - 1)], own = acc2[j];
      const bool sw = (unsigned)(t + FFT_M) < (unsigned)FFT_M;
      const uint32_t w0 = (t < 0) ? ~flip0 : flip0, w1 = (t < -FFT_M) ? ~flip0 : flip0;
      const uint32_t g0 = sw ? g.y : g.x, g1 = sw ? g.x : g.y;
      const uint32_t v0 = ((g0 ^ w0) - w0) - own.x;          // (+/- g0) - acc[j]
      const uint32_t v1 = ((g1 ^ w1) - w1) - own.y;
      // Balanced digit of the top base_log bits: arithmetic shift of the rounded 32-bit word.
      const int d0 = (int)(v0 + rnd) >> shift;
      const int d1 = (int)(v1 + rnd) >> shift;
      x[m] = make_double2((double)d0, (double)d1);
    }
    fft_forward_s<PNB_BR_CBANK>(x, buf, lane, wf_s);
    // GGSW i must have landed in shared memory (bounded wait; parity = i mod 2).
    if (!tc::mbar_wait(bar, (uint32_t)(i & 1), BR_WAIT_LIMIT)) {
      *abort_s = 1;
      atomicExch(&g_br_status, 1);
    }
    // Pointwise product in two halves of 16 registers, exchanged between the ciphertext's two
    // warps: output polynomial p = D_own * F[own row][p] + D_other * F[other row][p].
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) xbuf[rr * 32 + lane] = x[16 * h + rr];
      pair_sync(cl);
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) {
        const int r = 16 * h + rr;
        const int e = r * 32 + lane;
        const double2 fo = f_own[e], ft = f_oth[e];
        const double2 dt = obuf[rr * 32 + lane];
        const double2 p0 = cmul(x[r], fo);
        x[r] = make_double2(p0.x + fma(dt.x, ft.x, -dt.y * ft.y),
                            p0.y + fma(dt.x, ft.y, dt.y * ft.x));
      }
      pair_sync(cl);
    }
    // Every warp is done with GGSW i: stage GGSW i+1 while the inverse FFTs run.
    __syncthreads();
    if (*abort_s) {  // uniform: read by every thread after the same barrier
      // the copy of GGSW i may still be landing: let it (bounded) before the block exits
      if (threadIdx.x == 0) (void)tc::mbar_wait(bar, (uint32_t)(i & 1), BR_WAIT_LIMIT);
      break;
    }
    if (threadIdx.x == 0 && i + 1 < n) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      br_stage_ggsw(bsk_dst, fbsk + (size_t)(i + 1) * 4 * FFT_M, bar);
    }
    fft_inverse_s<10 + 32, PNB_BR_CBANK>(x, buf, lane, wf_s);
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if ((m & 7) == 0) asm volatile("" ::: "memory");
      const int j = lane + 32 * m;
      uint2 o = acc2[j];
      o.x += scaled_f64_to_top32(x[m].x);
      o.y += scaled_f64_to_top32(x[m].y);
      acc2[j] = o;
    }
    __syncwarp();
  }
  // Sample extraction of coefficient 0 into an LWE of dimension N under the big key.
  if (valid && !*abort_s) {
    uint64_t* o = out + (size_t)ct * out_ld;
    if (p == 0) {
      for (int t = lane; t < FFT_N; t += 32) {
        const uint64_t v = (uint64_t)acc_at(t == 0 ? 0 : FFT_N - t) << 32;
        o[t] = (t == 0) ? v : (uint64_t)0 - v;
      }
    } else if (lane == 0) {
      o[FFT_N] = (uint64_t)acc_at(0) << 32;
    }
  }
}

constexpr int BR_CPB = 4;

// ------------------------------------------------------------------------------------------
// The same blind rotation with the twiddles and the pair exchange in tensor memory.
//
// Shared memory serves every other stream of the CMux (digit formation, the two transposes, the
// key rows, the accumulator update); the forward and inverse twiddles (16 KB per warp and
// transform) and the exchange of the two warps' spectra (32 KB per warp and CMux) go through
// tensor memory instead, a third less shared-memory traffic.  Warp w owns polynomial
// p = w / 4 of ciphertext c = w % 4, so the two warps of a ciphertext share lane quarter c of
// tensor memory.  Columns (per lane quarter, lane l): [0, 128) forward twiddles T(r, l) for
// r = 0..31 as (re lo, re hi, im lo, im hi) words; [128, 256) T(l, n) for n = 0..31 (the inverse
// multiplies by their conjugates); [256, 384) and [384, 512) the spectra of the mask and body
// warps.
// ------------------------------------------------------------------------------------------
template <int CPB>
struct BrTmLayout {
  static constexpr int WARPS = 2 * CPB;
  static constexpr int SCRATCH = FFT_M * sizeof(double);            // 8 KB per warp
  static constexpr int ACC = FFT_N * sizeof(uint32_t);              // 8 KB per warp
  static constexpr int BSK = 4 * FFT_M * sizeof(double2);           // 64 KB: one GGSW (k=1,l=1)
  static constexpr int ABAR = BR_MAXN * sizeof(uint16_t);           // 2 KB per ciphertext
  static constexpr int OFF_ACC = WARPS * SCRATCH;
  static constexpr int OFF_BSK = OFF_ACC + WARPS * ACC;
  static constexpr int OFF_ABAR = OFF_BSK + BSK;
  static constexpr int OFF_BAR = OFF_ABAR + CPB * ABAR;  // mbarrier, abort flag, TMEM base
  static constexpr int BYTES = OFF_BAR + 16;
  static constexpr int TMEM_COLS = 512;
};

__device__ __forceinline__ void d2_to_words(double2 v, uint32_t* t) {
  t[0] = (uint32_t)__double2loint(v.x);
  t[1] = (uint32_t)__double2hiint(v.x);
  t[2] = (uint32_t)__double2loint(v.y);
  t[3] = (uint32_t)__double2hiint(v.y);
}
__device__ __forceinline__ double2 words_to_d2(const uint32_t* t) {
  return make_double2(__hiloint2double((int)t[1], (int)t[0]),
                      __hiloint2double((int)t[3], (int)t[2]));
}

// round(w) mod 2^32 for w = v 2^-32 (|w| < 2^63): with PNB_BR_F2I one conversion to a 64-bit
// integer (off the FP64 pipe), otherwise scaled_f64_to_top32's three FP64 operations.
#ifndef PNB_BR_F2I
#define PNB_BR_F2I 1
#endif
__device__ __forceinline__ uint32_t top32_round(double w) {
#if PNB_BR_F2I
  return (uint32_t)(unsigned long long)__double2ll_rn(w);
#else
  return scaled_f64_to_top32(w);
#endif
}
// Eight complex values (32 columns) per tensor-memory round trip: tcgen05.wait::ld waits for
// every load in flight, so a round trip is one load and one wait.
constexpr int BR_TC = 8;
__device__ __forceinline__ void tm_load8(uint32_t taddr, uint32_t (&t)[32]) {
  tc::tmem_ld_32x32_nowait(taddr, t);
  tc::tmem_ld_wait();
}

template <int CPB>
__global__ void __launch_bounds__(64 * CPB, 1) blind_rotate_tm_kernel(
    const uint64_t* __restrict__ small_ct, TvSel sel,
    const double2* __restrict__ fbsk, uint64_t* __restrict__ out, int out_ld, int count, int n,
    int base_log, FftTables tb) {
  static_assert(CPB == 4, "the lane-quarter mapping needs four ciphertexts per block");
  using L = BrTmLayout<CPB>;
  extern __shared__ __align__(128) unsigned char bt_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = warp & 3, p = warp >> 2;
  const int ct = blockIdx.x * CPB + cl;
  const bool valid = ct < count;
  constexpr int LG = 12;  // log2(2N)
  double* buf = reinterpret_cast<double*>(bt_raw) + warp * FFT_M;
  uint2* acc2 = reinterpret_cast<uint2*>(bt_raw + L::OFF_ACC) + warp * FFT_M;
  auto acc_at = [&](int e) { return e < FFT_M ? acc2[e].x : acc2[e - FFT_M].y; };
  const double2* bsk_s = reinterpret_cast<const double2*>(bt_raw + L::OFF_BSK);
  uint16_t* abar = reinterpret_cast<uint16_t*>(bt_raw + L::OFF_ABAR) + cl * BR_MAXN;
  const uint32_t bar = tc::smem_u32(bt_raw + L::OFF_BAR);
  volatile int* abort_s = reinterpret_cast<volatile int*>(bt_raw + L::OFF_BAR + 8);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bt_raw + L::OFF_BAR + 12);
  const uint32_t bsk_dst = tc::smem_u32(bt_raw + L::OFF_BSK);

  if (threadIdx.x == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
    *abort_s = 0;
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_u32(tmem_holder), L::TMEM_COLS);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (threadIdx.x == 0) br_stage_ggsw(bsk_dst, fbsk, bar);
  const uint32_t tq = *reinterpret_cast<volatile uint32_t*>(tmem_holder) +
                      ((uint32_t)(32 * cl) << 16);
  const uint32_t t_fwd = tq, t_inv = tq + 128u;
  const uint32_t t_own = tq + 256u + 128u * (uint32_t)p, t_oth = tq + 256u + 128u * (uint32_t)(p ^ 1);
  if (p == 0) {  // one warp per lane quarter writes its twiddles
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
      uint32_t t[16], u[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        d2_to_words(tb.wf[(4 * g + q) * 32 + lane], t + 4 * q);
        d2_to_words(tb.wf[lane * 32 + 4 * g + q], u + 4 * q);
      }
      tc::tmem_st_32x32_x16(t_fwd + 16u * g, t);
      tc::tmem_st_32x32_x16(t_inv + 16u * g, u);
    }
    tc::tmem_st_wait();
  }

  const uint64_t* in = small_ct + (size_t)(valid ? ct : 0) * (n + 1);
  const uint64_t* tv = tv_of(sel, valid ? ct : 0);
  const int t64 = lane + 32 * p;
  for (int i = t64; i < n; i += 64) abar[i] = valid ? (uint16_t)modswitch(in[i], LG) : 0;
  const int bt = valid ? modswitch(in[n], LG) : 0;
  const int r0 = (2 * FFT_N - bt) & (2 * FFT_N - 1);
  for (int t = lane; t < FFT_M; t += 32) {
    auto top = [&](int e) { return (uint32_t)((rot_coef(tv, e, r0) + 0x80000000ull) >> 32); };
    acc2[t] = (p == 0) ? make_uint2(0u, 0u) : make_uint2(top(t), top(t + FFT_M));
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();

  const int shift = 32 - base_log;
  const uint32_t rnd = 1u << (shift - 1);
  const double2* f_own = bsk_s + (size_t)(p * 2 + p) * FFT_M;
  const double2* f_oth = bsk_s + (size_t)((p ^ 1) * 2 + p) * FFT_M;

  // Each CMux interleaves integer or shared-memory work with FP64 butterflies in one instruction
  // stream: the digit formation with the forward transform's first pass (crt_dft32_from), the
  // products with the inverse transform's first four stages (per block of eight and per half),
  // and the accumulator update with its last stage (dit_dft32_untwist_to).  Every value meets
  // the same operations in the same order as in the plain transforms.
  for (int i = 0; i < n; ++i) {
    const int a = abar[i];
    const int ar = a & (FFT_N - 1);
    const uint32_t flip0 = (a >= FFT_N) ? 0xffffffffu : 0u;
    double2 x[FFT_R];
    // digits of (X^a - 1) acc for register m: coefficients lane + 32 m and lane + 32 m + M
    auto digit_pair = [&](int m) -> double2 {
      const int j = lane + 32 * m;
      const int t = j - ar;
      const uint2 g = acc2[t & (FFT_M - 1)], own = acc2[j];
      const bool sw = (unsigned)(t + FFT_M) < (unsigned)FFT_M;
      const uint32_t w0 = (t < 0) ? ~flip0 : flip0, w1 = (t < -FFT_M) ? ~flip0 : flip0;
      const uint32_t g0 = sw ? g.y : g.x, g1 = sw ? g.x : g.y;
      const uint32_t v0 = ((g0 ^ w0) - w0) - own.x;
      const uint32_t v1 = ((g1 ^ w1) - w1) - own.y;
      const int d0 = (int)(v0 + rnd) >> shift;
      const int d1 = (int)(v1 + rnd) >> shift;
      return make_double2((double)d0, (double)d1);
    };
    crt_dft32_from<32, PNB_BR_CBANK>(x, digit_pair);
    // the mid twiddles from tensor memory
#pragma unroll
    for (int g = 0; g < 32 / BR_TC; ++g) {
      uint32_t t[4 * BR_TC];
      tm_load8(t_fwd + 4u * BR_TC * g, t);
#pragma unroll
      for (int q = 0; q < BR_TC; ++q)
        x[BR_TC * g + q] = cmul(x[BR_TC * g + q], words_to_d2(t + 4 * q));
    }
    warp_transpose_half(x, buf, lane);
    crt_dft32<0, PNB_BR_CBANK>(x);
    // this warp's spectrum to tensor memory for the other warp of the ciphertext
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t t[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) d2_to_words(x[4 * g + q], t + 4 * q);
      tc::tmem_st_32x32_x16(t_own + 16u * g, t);
    }
    tc::tmem_st_wait();
    // GGSW i must have landed in shared memory (bounded wait; parity = i mod 2).
    if (!tc::mbar_wait(bar, (uint32_t)(i & 1), BR_WAIT_LIMIT)) {
      *abort_s = 1;
      atomicExch(&g_br_status, 1);
    }
    tc::tc_fence_before();
    pair_sync(cl);
    tc::tc_fence_after();
    // output polynomial p = D_own * F[own row][p] + D_other * F[other row][p], then the inverse
    // transform's stages 1-3 per block of eight registers and stage 4 per half of sixteen
#pragma unroll
    for (int g = 0; g < 32 / BR_TC; ++g) {
      uint32_t t[4 * BR_TC];
      tm_load8(t_oth + 4u * BR_TC * g, t);
#pragma unroll
      for (int q = 0; q < BR_TC; ++q) {
        const int r = BR_TC * g + q;
        const int e = r * 32 + lane;
        const double2 fo = f_own[e], ft = f_oth[e];
        const double2 dt = words_to_d2(t + 4 * q);
        // x fo + dt ft as one chain of fused multiply-adds per component (8 FP64 operations)
        const double2 xv = x[r];
        x[r] = make_double2(fma(xv.x, fo.x, fma(-xv.y, fo.y, fma(dt.x, ft.x, -dt.y * ft.y))),
                            fma(xv.x, fo.y, fma(xv.y, fo.x, fma(dt.x, ft.y, dt.y * ft.x))));
      }
      dit_block8<PNB_BR_CBANK>(x, g);
      if (g & 1) {  // dit_stage<4> on registers 16 (g >> 1) .. + 15
        const int s0 = 16 * (g >> 1);
#pragma unroll
        for (int j = 0; j < 8; ++j) ct_bfly<PNB_BR_CBANK>(128 - 8 * j, x[s0 + j], x[s0 + j + 8]);
      }
    }
    // Every warp is done with GGSW i and with the other warp's spectrum: stage GGSW i+1 while
    // the inverse transforms run.
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (*abort_s) {  // uniform: read by every thread after the same barrier
      if (threadIdx.x == 0) (void)tc::mbar_wait(bar, (uint32_t)(i & 1), BR_WAIT_LIMIT);
      break;
    }
    if (threadIdx.x == 0 && i + 1 < n) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      br_stage_ggsw(bsk_dst, fbsk + (size_t)(i + 1) * 4 * FFT_M, bar);
    }
    // inverse transform: its last first-pass stage, the conjugate twiddles from tensor memory
    dit_stage<5, PNB_BR_CBANK>(x);
#pragma unroll
    for (int g = 0; g < 32 / BR_TC; ++g) {
      uint32_t t[4 * BR_TC];
      tm_load8(t_inv + 4u * BR_TC * g, t);
#pragma unroll
      for (int q = 0; q < BR_TC; ++q)
        x[BR_TC * g + q] = cmul_conj(x[BR_TC * g + q], words_to_d2(t + 4 * q));
    }
    warp_transpose_half(x, buf, lane);
    // acc += round(inverse transform), register m = coefficients lane + 32 m and lane + 32 m + M
    dit_dft32_untwist_to<10 + 32, PNB_BR_CBANK>(x, [&](int m) {
      const int j = lane + 32 * m;
      uint2 o = acc2[j];
      o.x += top32_round(x[m].x);
      o.y += top32_round(x[m].y);
      acc2[j] = o;
    });
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(*reinterpret_cast<volatile uint32_t*>(tmem_holder), L::TMEM_COLS);
  }
  // Sample extraction of coefficient 0 into an LWE of dimension N under the big key.
  if (valid && !*abort_s) {
    uint64_t* o = out + (size_t)ct * out_ld;
    if (p == 0) {
      for (int t = lane; t < FFT_N; t += 32) {
        const uint64_t v = (uint64_t)acc_at(t == 0 ? 0 : FFT_N - t) << 32;
        o[t] = (t == 0) ? v : (uint64_t)0 - v;
      }
    } else if (lane == 0) {
      o[FFT_N] = (uint64_t)acc_at(0) << 32;
    }
  }
}

// Which single-level rotation runs: 1 = twiddles and exchange in tensor memory, 0 = in shared
// memory.
#ifndef PNB_BR_TMEM
#define PNB_BR_TMEM 1
#endif

// ------------------------------------------------------------------------------------------
// Blocked multi-level blind rotation (pbs_level 2..6).  A block bootstraps MLB_CPB ciphertexts
// in lockstep, warp (2c + p) owning accumulator polynomial p of ciphertext c, like the single-
// level kernel; per CMux it walks the gadget levels, and each level's part of the GGSW (the mask
// and body rows of that level, 64 KB) is staged once per block in shared memory by bulk copy
// while the warps form and transform the level's digits, so the ciphertexts of a block share
// every key byte.  Tensor memory holds, per warp, the sums of levels 0..L-2 (128 columns; the
// last level's sum stays in registers and goes through the inverse transform) and the rounded,
// offset coefficient differences the first level computes from the accumulator (128 columns),
// from which every later level reads its digits with a shift and a mask; warps w and w + 4 share
// a lane quarter, so the block takes all 512 columns.  The accumulator keeps the top 48 bits of each torus coefficient (u64
// words whose low 16 bits stay zero): the gadget digits read at most 42 bits plus a rounding
// bit, and the dropped bits (< 2^16 per CMux) stay far below the f64 product's own error.
// ------------------------------------------------------------------------------------------
constexpr int MLB_CPB = 4;

struct MlbLayout {
  static constexpr int WARPS = 2 * MLB_CPB;
  static constexpr int SCRATCH = FFT_M * sizeof(double);      // 8 KB per warp
  static constexpr int ACC_HI = FFT_N * sizeof(uint32_t);     // 8 KB per warp: bits 32..63
  static constexpr int ACC_LO = FFT_N * sizeof(uint16_t);     // 4 KB per warp: bits 16..31
  static constexpr int GGSW = 4 * FFT_M * sizeof(double2);    // 64 KB: one level
  static constexpr int OFF_HI = WARPS * SCRATCH;
  static constexpr int OFF_LO = OFF_HI + WARPS * ACC_HI;
  static constexpr int OFF_GGSW = OFF_LO + WARPS * ACC_LO;
  static constexpr int OFF_BAR = OFF_GGSW + GGSW;  // mbarrier, abort flag, TMEM base
  static constexpr int BYTES = OFF_BAR + 16;
  static constexpr int TMEM_COLS = 512;  // per warp: 128 level-sum + 128 digit-source columns
};

// w = v 2^-16 for the exact product coefficient v (|w| < 2^86).  Returns round(w) mod 2^48 in the
// top 48 bits of a torus word, with three FP64 operations: with C = 1.5 * 2^52,
// u = RN(w 2^-48 + C) = C + k, k = round(w / 2^48); q = C (1 + 2^48) - 2^48 u = C - 2^48 k
// exactly; w + q = (w - 2^48 k) + C with |w - 2^48 k| <= 2^47, so its rounding to the unit grid of
// [2^52, 2^53) is C + round(w - 2^48 k), and the low 48 bits of that double's encoding are
// round(w) mod 2^48 (C's mantissa 2^51 is 0 mod 2^48).
__device__ __forceinline__ uint64_t scaled_f64_to_top48(double w) {
  const double magic = 6755399441055744.0;                    // 1.5 * 2^52
  const double magic_hi = 6755399441055744.0 * 281474976710657.0;  // C (1 + 2^48), exact
  const double u = fma(w, 0x1p-48, magic);
  const double q = fma(u, -281474976710656.0, magic_hi);
  return (uint64_t)__double_as_longlong(w + q) << 16;
}

// Stage level `lev` of GGSW `i` (key set with L levels): the mask row's two polynomials to slots
// 0..1 and the body row's to slots 2..3 (64 KB).
template <int L>
__device__ __forceinline__ void mlb_stage(uint32_t dst, const double2* fbsk, int i, int lev,
                                          uint32_t bar) {
  const double2* g = fbsk + (size_t)i * (2 * L) * 2 * FFT_M;
  tc::mbar_expect_tx(bar, 4 * FFT_M * sizeof(double2));
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int row = (q < 2 ? 0 : L) + lev;
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst + q * FFT_M * 16u), "l"(g + (size_t)(row * 2 + (q & 1)) * FFT_M),
        "r"(FFT_M * 16u), "r"(bar)
        : "memory");
  }
}

template <int L, int BETA>
__global__ void __launch_bounds__(64 * MLB_CPB, 1) blind_rotate_mlb_kernel(
    const uint64_t* __restrict__ small_ct, TvSel sel, const double2* __restrict__ fbsk,
    uint64_t* __restrict__ out, int out_ld, int count, int n, int base_log, FftTables tb) {
  using Y = MlbLayout;
  extern __shared__ __align__(128) unsigned char mlb_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = warp >> 1, p = warp & 1;
  const int ct = blockIdx.x * MLB_CPB + cl;
  const bool valid = ct < count;
  constexpr int LG = 12;  // log2(2N)
  double* buf = reinterpret_cast<double*>(mlb_raw) + warp * FFT_M;
  double2* xch = reinterpret_cast<double2*>(buf);
  const double2* och = reinterpret_cast<const double2*>(reinterpret_cast<double*>(mlb_raw) +
                                                        (warp ^ 1) * FFT_M);
  // accumulator word t = hi[t] 2^32 + lo[t] 2^16 (the low 16 bits stay zero)
  // with coefficients (j, j + M) side by side: hi2[j] = (hi[j], hi[j + M]), lo2 likewise.
  // A32: when the digits read at most 30 bits (beta L <= 30) only hi is kept -- the top 32 bits,
  // as in the single-level kernel (the dropped word adds a random walk of ~2^36 against these
  // key sets' 2^41 and more of output noise).
  constexpr bool A32 = BETA > 0 && BETA * L <= 30;
  uint2* hi2 = reinterpret_cast<uint2*>(mlb_raw + Y::OFF_HI) + warp * FFT_M;
  ushort2* lo2 = reinterpret_cast<ushort2*>(mlb_raw + Y::OFF_LO) + warp * FFT_M;
  auto word = [](uint32_t hi, uint16_t lo) {
    return ((uint64_t)hi << 32) | (A32 ? 0ull : (uint64_t)lo << 16);
  };
  auto acc_at = [&](int e) {
    return e < FFT_M ? word(hi2[e].x, A32 ? 0 : lo2[e].x)
                     : word(hi2[e - FFT_M].y, A32 ? 0 : lo2[e - FFT_M].y);
  };
  auto acc_put2 = [&](int k, uint64_t v0, uint64_t v1) {
    hi2[k] = make_uint2((uint32_t)(v0 >> 32), (uint32_t)(v1 >> 32));
    if (!A32) lo2[k] = make_ushort2((uint16_t)(v0 >> 16), (uint16_t)(v1 >> 16));
  };
  const double2* ggsw_s = reinterpret_cast<const double2*>(mlb_raw + Y::OFF_GGSW);
  const uint32_t bar = tc::smem_u32(mlb_raw + Y::OFF_BAR);
  volatile int* abort_s = reinterpret_cast<volatile int*>(mlb_raw + Y::OFF_BAR + 8);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mlb_raw + Y::OFF_BAR + 12);
  const uint32_t ggsw_dst = tc::smem_u32(mlb_raw + Y::OFF_GGSW);

  if (threadIdx.x == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
    *abort_s = 0;
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_u32(tmem_holder), Y::TMEM_COLS);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (threadIdx.x == 0) mlb_stage<L>(ggsw_dst, fbsk, 0, 0, bar);

  const uint64_t* in = small_ct + (size_t)(valid ? ct : 0) * (n + 1);
  const uint64_t* tv = tv_of(sel, valid ? ct : 0);
  const int bt = valid ? modswitch(in[n], LG) : 0;
  const int r0 = (2 * FFT_N - bt) & (2 * FFT_N - 1);
  for (int t = lane; t < FFT_M; t += 32) {
    // A32 keeps the rounded top word (as the single-level kernel does)
    auto init = [&](int e) {
      const uint64_t v = (p == 0) ? 0 : rot_coef(tv, e, r0);
      return A32 ? (v + 0x80000000ull) & ~0xffffffffull : v;
    };
    acc_put2(t, init(t), init(t + FFT_M));
  }
  uint64_t a_next = valid ? in[0] : 0;  // mask coefficient of the next CMux, loaded one ahead
  __syncthreads();

  // this warp's lane quarter and column range; column 4r + {0..3} holds spectrum row r.  The
  // 32-bit form keeps one vk word per coefficient (64 columns per warp), and the forward
  // transform's twiddles T(r, lane) take the quarter's last 128 columns.
  const uint32_t tq = *reinterpret_cast<volatile uint32_t*>(tmem_holder) +
                      ((uint32_t)(32 * (warp & 3)) << 16);
  const uint32_t tfacc = tq + (uint32_t)(128 * (warp >> 2));
  const uint32_t tvk = A32 ? tq + 256u + (uint32_t)(64 * (warp >> 2)) : tfacc + 256u;
  const uint32_t t_fwd = tq + 384u;
  if (A32 && warp < 4) {  // one warp per lane quarter writes its twiddles
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
      uint32_t t[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) d2_to_words(tb.wf[(4 * g + q) * 32 + lane], t + 4 * q);
      tc::tmem_st_32x32_x16(t_fwd + 16u * g, t);
    }
    tc::tmem_st_wait();
    tc::tc_fence_before();
  }
  __syncthreads();
  tc::tc_fence_after();
  const double2* f_own = ggsw_s + (size_t)(p * 2 + p) * FFT_M;
  const double2* f_oth = ggsw_s + (size_t)((p ^ 1) * 2 + p) * FFT_M;
  // Gadget digits: with T = beta L and H = sum_j 2^(beta-1) 2^(beta j), the balanced digits of
  // the top T bits of v, rounded, are the plain base-2^beta digits of round(v / 2^(64-T)) + H,
  // each minus 2^(beta-1); that sum is the top T bits of vk = v + vk_off (mod 2^64) with
  // vk_off = 2^(63-T) + H 2^(64-T), the rounding folded into the carry.
  const int beta = BETA > 0 ? BETA : base_log;
  uint64_t hsum = 0;
#pragma unroll
  for (int j = 0; j < L; ++j) hsum |= (1ull << (beta - 1)) << (beta * j);
  const uint64_t vk_off = (1ull << (63 - beta * L)) + (hsum << (64 - beta * L));
  const uint32_t dmask = (1u << beta) - 1u;
  const int dhalf = 1 << (beta - 1);
  // A32: the digit source is the top word; the rounding unit is bit 32 - T of it, and ties are
  // broken to even by adding half a unit less one plus the lowest kept bit
  const int rnd_sh = A32 ? 32 - beta * L : 1;
  const uint32_t off_h = A32 ? (uint32_t)(vk_off >> 32) - 1u : 0u;
  uint32_t stage = 0;
  bool aborted = false;

  for (int i = 0; i < n && !aborted; ++i) {
    const int a = modswitch(a_next, LG);
    if (valid && i + 1 < n) a_next = in[i + 1];
    double2 x[FFT_R];
    {
      // vk = (X^a acc - acc) + vk_off for both halves of every coefficient pair, into tensor
      // memory (four columns per register pair); X^a = (-1)^(a >= N) X^(a mod N): rotate by ar
      // in [0, N) and flip the sign where the rotation wraps.
      const int ar = a & (FFT_N - 1);
      const uint64_t flip = (a >= FFT_N) ? ~0ull : 0ull;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        uint32_t t[16], u[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = lane + 32 * (4 * g + q);
          // coefficients t = j - ar and t + M of X^ar acc share the pair slot t mod M: t >= 0
          // reads (x, y) as they are, -M <= t < 0 reads (-y, x), t < -M reads (-x, -y)
          const int tr = j - ar;
          const uint2 gh = hi2[tr & (FFT_M - 1)], oh = hi2[j];
          const bool sw = (unsigned)(tr + FFT_M) < (unsigned)FFT_M;
          if (A32) {
            // The same in 32-bit words, vk in the top word.  With no bits below the word,
            // exact ties of the rounding (v mod 2^(33-T+32) = half a unit) are common, and
            // rounding them all up would bias every coefficient by half a word -- a bias the
            // external product sums coherently over the key.  Ties go to the even value.
            const uint32_t f32 = (uint32_t)flip;
            const uint32_t n0 = (tr < 0 ? ~0u : 0u) ^ f32, n1 = (tr < -FFT_M ? ~0u : 0u) ^ f32;
            const uint32_t g0 = sw ? gh.y : gh.x, g1 = sw ? gh.x : gh.y;
            const uint32_t w0 = ((g0 ^ n0) - n0) - oh.x, w1 = ((g1 ^ n1) - n1) - oh.y;
            u[2 * q + 0] = w0 + off_h + ((w0 >> rnd_sh) & 1u);
            u[2 * q + 1] = w1 + off_h + ((w1 >> rnd_sh) & 1u);
          } else {
            const ushort2 gl = lo2[tr & (FFT_M - 1)], ol = lo2[j];
            const uint64_t n0 = (tr < 0 ? ~0ull : 0ull) ^ flip;
            const uint64_t n1 = (tr < -FFT_M ? ~0ull : 0ull) ^ flip;
            const uint64_t ga = word(gh.x, gl.x), gb = word(gh.y, gl.y);
            const uint64_t g0 = sw ? gb : ga, g1 = sw ? ga : gb;
            const uint64_t v0 = ((g0 ^ n0) - n0) - word(oh.x, ol.x) + vk_off;
            const uint64_t v1 = ((g1 ^ n1) - n1) - word(oh.y, ol.y) + vk_off;
            t[4 * q + 0] = (uint32_t)v0;
            t[4 * q + 1] = (uint32_t)(v0 >> 32);
            t[4 * q + 2] = (uint32_t)v1;
            t[4 * q + 3] = (uint32_t)(v1 >> 32);
          }
        }
        if (A32) tc::tmem_st_32x32_x8(tvk + (uint32_t)(8 * g), u);
        else tc::tmem_st_32x32_x16(tvk + (uint32_t)(16 * g), t);
      }
      tc::tmem_st_wait();
    }
#pragma unroll 1
    for (int lev = 0; lev < L; ++lev) {
      // digit `lev` sits in bits [sh, sh + beta) of vk: a funnel shift by min(sh, 32), then sh - 32
      const int sh = 64 - beta * (lev + 1);
      const int sh_a = sh < 32 ? sh : 32, sh_b = sh - sh_a;
      if (A32) {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint32_t u[8];
          tc::tmem_ld_32x32_x8(tvk + (uint32_t)(8 * g), u);
          tc::tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int d = (int)((u[q] >> (sh - 32)) & dmask) - dhalf;
            if (q & 1) x[4 * g + (q >> 1)].y = (double)d;
            else x[4 * g + (q >> 1)].x = (double)d;
          }
        }
        // forward transform with the mid twiddles from tensor memory
        crt_dft32<32, PNB_ML_CBANK>(x);
#pragma unroll
        for (int g = 0; g < 32 / BR_TC; ++g) {
          uint32_t t[4 * BR_TC];
          tm_load8(t_fwd + 4u * BR_TC * g, t);
#pragma unroll
          for (int q = 0; q < BR_TC; ++q)
            x[BR_TC * g + q] = cmul(x[BR_TC * g + q], words_to_d2(t + 4 * q));
        }
        warp_transpose_half(x, buf, lane);
        crt_dft32<0, PNB_ML_CBANK>(x);
      } else {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint32_t t[16];
          tc::tmem_ld_32x32_x16(tvk + (uint32_t)(16 * g), t);
          tc::tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int d =
                (int)((__funnelshift_rc(t[2 * q], t[2 * q + 1], sh_a) >> sh_b) & dmask) - dhalf;
            if (q & 1) x[4 * g + (q >> 1)].y = (double)d;
            else x[4 * g + (q >> 1)].x = (double)d;
          }
        }
        fft_forward_h<PNB_ML_CBANK>(x, buf, lane, tb.wf);
      }
      // this level's key rows must have landed (bounded wait; parity = stage mod 2)
      if (!tc::mbar_wait(bar, stage & 1u, BR_WAIT_LIMIT)) {
        *abort_s = 1;
        atomicExch(&g_br_status, 1);
      }
      const bool last = lev == L - 1;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) xch[rr * 32 + lane] = x[16 * h + rr];
        pair_sync(cl);
#pragma unroll
        for (int g8 = 0; g8 < 2; ++g8) {
          const int rb = 16 * h + 8 * g8;  // eight spectrum rows = 32 TMEM columns
          uint32_t t[32];
          if (lev > 0) {
            tc::tmem_ld_32x32_nowait(tfacc + (uint32_t)(4 * rb), t);
            tc::tmem_ld_wait();
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int r = rb + q;
            const int e = r * 32 + lane;
            const double2 fo = f_own[e], ft = f_oth[e];
            const double2 dt = och[(r - 16 * h) * 32 + lane];
            // x fo + dt ft (+ the earlier levels' sum) as one chain of fused multiply-adds
            const double2 sum = lev > 0 ? words_to_d2(t + 4 * q) : make_double2(0.0, 0.0);
            const double2 xv = x[r];
            const double2 v =
                make_double2(fma(xv.x, fo.x, fma(-xv.y, fo.y, fma(dt.x, ft.x, fma(-dt.y, ft.y, sum.x)))),
                             fma(xv.x, fo.y, fma(xv.y, fo.x, fma(dt.x, ft.y, fma(dt.y, ft.x, sum.y)))));
            if (last) {
              x[r] = v;
            } else {
              d2_to_words(v, t + 4 * q);
            }
          }
          if (!last) tc::tmem_st_32x32(tfacc + (uint32_t)(4 * rb), t);
        }
        pair_sync(cl);
      }
      if (!last) tc::tmem_st_wait();
      // every warp is done with this level's key rows: stage the next level (or the next CMux's
      // first level) while the warps carry on
      __syncthreads();
      if (*abort_s) {  // uniform: read by every thread after the same barrier
        aborted = true;
        break;
      }
      ++stage;
      if (threadIdx.x == 0 && (i + 1 < n || lev + 1 < L)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (lev + 1 < L) mlb_stage<L>(ggsw_dst, fbsk, i, lev + 1, bar);
        else mlb_stage<L>(ggsw_dst, fbsk, i + 1, 0, bar);
      }
    }
    if (aborted) break;
    fft_inverse_h<PNB_ML_CBANK, A32 ? 10 + 32 : 10 + 16>(x, buf, lane, tb.wi);
    // acc += round(inverse transform): the 32-bit form by one 64-bit conversion (|w| < 2^63),
    // the 48-bit form by three FP64 operations (|w| reaches past 2^63)
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if ((m & 7) == 0) asm volatile("" ::: "memory");
      const int j = lane + 32 * m;
      if (A32) {
        uint2 h = hi2[j];
        h.x += top32_round(x[m].x);
        h.y += top32_round(x[m].y);
        hi2[j] = h;
      } else {
        const uint2 h = hi2[j];
        const ushort2 l = lo2[j];
        acc_put2(j, word(h.x, l.x) + scaled_f64_to_top48(x[m].x),
                 word(h.y, l.y) + scaled_f64_to_top48(x[m].y));
      }
    }
    __syncwarp();
  }
  if (aborted && threadIdx.x == 0) {
    // a copy of the stage that timed out may still be in flight: let it land (bounded) before
    // the block's shared memory is released
    (void)tc::mbar_wait(bar, stage & 1u, BR_WAIT_LIMIT);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(*reinterpret_cast<volatile uint32_t*>(tmem_holder), Y::TMEM_COLS);
  }
  // Sample extraction of coefficient 0 into an LWE of dimension N under the big key.
  if (valid && !aborted) {
    uint64_t* o = out + (size_t)ct * out_ld;
    if (p == 0) {
      for (int t = lane; t < FFT_N; t += 32)
        o[t] = (t == 0) ? acc_at(0) : (uint64_t)0 - acc_at(FFT_N - t);
    } else if (lane == 0) {
      o[FFT_N] = acc_at(0);
    }
  }
}

template <int L, int BETA>
static int launch_mlb(const pnb_keys* K, TvSel tv, const uint64_t* small, uint64_t* out,
                      int out_ld, int count, FftTables tb, cudaStream_t st) {
  constexpr int smem = MlbLayout::BYTES;
  PNB_CUDA(cudaFuncSetAttribute(blind_rotate_mlb_kernel<L, BETA>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int blocks = (count + MLB_CPB - 1) / MLB_CPB;
  blind_rotate_mlb_kernel<L, BETA><<<blocks, 64 * MLB_CPB, smem, st>>>(
      small, tv, K->fbsk, out, out_ld, count, K->p.n, K->p.pbs_base_log, tb);
  PNB_CHECK_LAUNCH("blind_rotate_mlb_kernel");
  return PNB_OK;
}

// The key sets the graph planner uses get kernels with compile-time gadget constants.
template <int L, int B0, int B1 = 0>
static int launch_ml_any(const pnb_keys* K, TvSel tv, const uint64_t* small, uint64_t* out,
                         int out_ld, int count, FftTables tb, cudaStream_t st) {
  if (B0 > 0 && K->p.pbs_base_log == B0)
    return launch_mlb<L, B0>(K, tv, small, out, out_ld, count, tb, st);
  if (B1 > 0 && K->p.pbs_base_log == B1)
    return launch_mlb<L, B1>(K, tv, small, out, out_ld, count, tb, st);
  return launch_mlb<L, 0>(K, tv, small, out, out_ld, count, tb, st);
}

static bool br_supported(const pnb_params& p) {
  if (p.N == 8192) return br8k_supported(p);
  if (p.k != 1 || p.N != FFT_N || p.n > BR_MAXN || p.n <= 0) return false;
  if (p.pbs_level == 1) return p.pbs_base_log >= 2 && p.pbs_base_log <= 30;
  // multi-level: digits below 2^22 in magnitude keep the f64 product's error small, and the
  // 48-bit accumulator holds the digits' T = base_log * level bits plus the rounding bit
  if (p.pbs_level == 9) return p.pbs_base_log == 5;
  return p.pbs_level >= 2 && p.pbs_level <= 6 && p.pbs_base_log >= 2 &&
         p.pbs_base_log <= 22 && p.pbs_base_log * p.pbs_level <= 46;
}

int blind_rotate_launch(const pnb_keys* K, const uint64_t* tv, const uint64_t* small,
                        uint64_t* out, int count, cudaStream_t st) {
  return blind_rotate_sel(K, tv, nullptr, 1, 0, small, out, count, st);
}

int blind_rotate_sel(const pnb_keys* K, const uint64_t* tvs, const int32_t* tv_idx, int period,
                     int first, const uint64_t* small, uint64_t* out, int count, cudaStream_t st,
                     int out_ld) {
  if (tv_idx && (period <= 0 || first < 0)) {
    set_error("blind rotation: test-vector period must be positive");
    return PNB_ERR_INVALID;
  }
  if (K->p.N == 8192)
    return blind_rotate_8k(K, tvs, tv_idx, period, tv_idx ? first % period : 0, small, out,
                           out_ld == 0 ? K->p.N + 1 : out_ld, count, st);
  const TvSel tv{tvs, tv_idx, period, tv_idx ? first % period : 0};
  if (!br_supported(K->p)) {
    set_error("blind rotation: compiled kernels cover k=1 with N=2048 (pbs_level 1..6 and "
              "(2^5, 9), n<=%d) or N=8192 ((2^23, 1), (2^15, 2), (2^11, 4)) (got "
              "k=%d N=%d level=%d base_log=%d n=%d)", BR_MAXN, K->p.k, K->p.N, K->p.pbs_level,
              K->p.pbs_base_log, K->p.n);
    return PNB_ERR_UNSUPPORTED;
  }
  if (out_ld == 0) out_ld = FFT_N + 1;
  if (out_ld < FFT_N + 1) {
    set_error("blind rotation: output row pitch %d is shorter than %d words", out_ld, FFT_N + 1);
    return PNB_ERR_INVALID;
  }
  if (count <= 0) return PNB_OK;
  FftTables tb;
  int rc = fft_tables_get(&tb);
  if (rc) return rc;
  switch (K->p.pbs_level) {
    case 1: break;
    case 2: return launch_ml_any<2, 15>(K, tv, small, out, out_ld, count, tb, st);
    case 3: return launch_ml_any<3, 11>(K, tv, small, out, out_ld, count, tb, st);
    case 4: return launch_ml_any<4, 10>(K, tv, small, out, out_ld, count, tb, st);
    case 5: return launch_ml_any<5, 8>(K, tv, small, out, out_ld, count, tb, st);
    case 6: return launch_ml_any<6, 7>(K, tv, small, out, out_ld, count, tb, st);
    case 9: return launch_mlb<9, 5>(K, tv, small, out, out_ld, count, tb, st);
    default:
      set_error("blind rotation: pbs_level %d not compiled", K->p.pbs_level);
      return PNB_ERR_UNSUPPORTED;
  }
  const int blocks = (count + BR_CPB - 1) / BR_CPB;
#if PNB_BR_TMEM
  constexpr int smem = BrTmLayout<BR_CPB>::BYTES;
  PNB_CUDA(cudaFuncSetAttribute(blind_rotate_tm_kernel<BR_CPB>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  blind_rotate_tm_kernel<BR_CPB><<<blocks, 64 * BR_CPB, smem, st>>>(
      small, tv, K->fbsk, out, out_ld, count, K->p.n, K->p.pbs_base_log, tb);
  PNB_CHECK_LAUNCH("blind_rotate_tm_kernel");
#else
  constexpr int smem = BrLayout<BR_CPB>::BYTES;
  PNB_CUDA(cudaFuncSetAttribute(blind_rotate_kernel<BR_CPB>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  blind_rotate_kernel<BR_CPB><<<blocks, 64 * BR_CPB, smem, st>>>(
      small, tv, K->fbsk, out, out_ld, count, K->p.n, K->p.pbs_base_log, tb);
  PNB_CHECK_LAUNCH("blind_rotate_kernel");
#endif
  return PNB_OK;
}

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

size_t pbs_workspace_bytes(const pnb_keys* K, int count) {
  if (!K || count <= 0) return 0;
  return align256((size_t)count * (K->p.n + 1) * sizeof(uint64_t)) +
         ks_tc_workspace_bytes(K->p, count);
}

int pbs_batch(const pnb_keys* K, const uint64_t* tv, const uint64_t* in, uint64_t* out,
              int count, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!br_supported(K->p)) {
    set_error("pbs: compiled kernels cover k=1 with N=2048 (pbs_level 1..6 and (2^5, 9), "
              "n<=%d) or N=8192 ((2^23, 1), (2^15, 2), (2^11, 4)) (got k=%d N=%d "
              "level=%d base_log=%d n=%d)", BR_MAXN, K->p.k, K->p.N, K->p.pbs_level,
              K->p.pbs_base_log, K->p.n);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count == 0) return PNB_OK;
  int rc = PNB_OK;
  const size_t need = pbs_workspace_bytes(K, count);
  unsigned char* w = nullptr;
  bool own = false;
  if (ws) {
    if (ws_bytes < need) {
      set_error("pbs: workspace of %zu bytes is smaller than the %zu bytes needed", ws_bytes,
                need);
      return PNB_ERR_INVALID;
    }
    if ((uintptr_t)ws % 256 != 0) {
      set_error("pbs: workspace must be 256-byte aligned");
      return PNB_ERR_INVALID;
    }
    w = static_cast<unsigned char*>(ws);
  } else {
    cudaError_t e = cudaMallocAsync((void**)&w, need, st);
    if (e != cudaSuccess) return cuda_status(e, "cudaMallocAsync(pbs workspace)");
    own = true;
  }
  uint64_t* small = reinterpret_cast<uint64_t*>(w);
  void* digits = w + align256((size_t)count * (K->p.n + 1) * sizeof(uint64_t));
  rc = keyswitch_launch(K, in, small, count, digits, st);
  if (rc == PNB_OK) rc = blind_rotate_launch(K, tv, small, out, count, st);
  if (own) {
    cudaError_t e = cudaFreeAsync(w, st);
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
  if (N == 8192) return fft_negacyclic_mul_8k(a, b, out, count, st);
  if (N != FFT_N) {
    set_error("fft_negacyclic_mul: compiled for N = %d and 8192, got %d", FFT_N, N);
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
