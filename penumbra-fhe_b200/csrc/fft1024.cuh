// fft1024.cuh -- warp-level negacyclic FFT for polynomials of size N = 2048.
//
// A real polynomial a(X) mod X^N + 1 is folded into M = N/2 complex coefficients
//   y_j = a_j + i a_{j+M},
// and the transform evaluates y at the M roots rho of X^M = i (a(rho) = y(rho) there; the other
// half of the roots of X^N + 1 are their conjugates, redundant for a real a).  Products of such
// evaluations are negacyclic products.  This is the "folding" evaluation tfhe-rs performs with
// its f64 FFT (tfhe-fft 0.10.1), restated for one warp:
//
//   M = 1024 = 32 x 32.  Lane l holds y_{l + 32 m} in register m.
//   forward : per lane, the 32-point evaluation of sum_m y_{l+32m} X^m at the 32 roots sigma_r of
//             X^32 = i, by the Cooley-Tukey reduction tree X^32 - i -> (X^16 - s)(X^16 + s) ...
//             (natural input, roots in bit-reversed order; the twist by the 1024th root is part
//             of the tree's twiddles) -> twiddle rho_r^l, rho_r = exp(i pi (1 + 4 br(r)) / 2048)
//             -> shared-memory transpose -> the same tree for X^32 - 1.  Result: lane r,
//             register s holds y(rho_r w^br(s)), w = exp(2 pi i / 32), br = 5-bit reversal.
//   inverse : per lane, a decimation-in-time DFT32 (bit-reversed input, natural output) ->
//             conjugate twiddle -> transpose -> DFT32 -> untwist exp(-i pi m / 64) / 1024.
//
// Every butterfly has the form (u + w v, u - w v) with the twiddle w ahead of the sum, so each
// one with a non-trivial w is six FMAs (Linzer-Feig: w v = A v (1 + iB) or A v (B + i)); a
// butterfly with w in {1, i, -1, -i} is four adds.  No bit reversal is materialised: pointwise
// products happen in the spectrum order above, and the Fourier bootstrapping key is produced by
// the same forward routine.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "fft_consts.cuh"

namespace pnb {

constexpr int FFT_R = 32;       // registers (complex) per lane
constexpr int FFT_M = 1024;     // complex points per polynomial
constexpr int FFT_N = 2048;     // polynomial size

// Twiddle tables between the two 32-point passes (device global memory, one set per device).
struct FftTables {
  double2* wf;  // [r*32 + l] = T(r, l) = rho_r^l                 (forward: lane l, register r)
  double2* wi;  // [n*32 + l] = conj(T(l, n))                      (inverse: lane l, register n)
};

__host__ __device__ constexpr int bitrev_bits(int v, int bits) {
  int r = 0;
  for (int b = 0; b < bits; ++b)
    if (v & (1 << b)) r |= 1 << (bits - 1 - b);
  return r;
}

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
  return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
// a * conj(b)
__device__ __forceinline__ double2 cmul_conj(double2 a, double2 b) {
  return make_double2(fma(a.x, b.x, a.y * b.y), fma(a.y, b.x, -a.x * b.y));
}

// (u, v) <- (u + w v, u - w v), w = exp(2 pi i e / 128).  `e` is a compile-time constant after
// unrolling, so every branch below folds away.  CB selects where the factors come from: the
// constant bank (operands of the FMAs themselves) or literals (materialised in uniform
// registers); which one leaves fewer general registers live depends on the kernel around it.
template <bool CB>
__device__ __forceinline__ void ct_bfly(int e, double2& u, double2& v) {
  e &= 127;
  double px, py;  // w v, or w v / A in the fused forms
  if (e % 32 == 0) {
    if (e == 0) { px = v.x; py = v.y; }
    else if (e == 32) { px = -v.y; py = v.x; }
    else if (e == 64) { px = -v.x; py = -v.y; }
    else { px = v.y; py = -v.x; }
    const double2 a = u;
    u = make_double2(a.x + px, a.y + py);
    v = make_double2(a.x - px, a.y - py);
    return;
  }
  double A, B;
  if (CB) {
    A = kLF128[e].x;
    B = kLF128[e].y;
  } else {
    lf128_lit(e, A, B);
  }
  if (lf_tan_form(e)) {  // w v = A (v.x - B v.y, v.y + B v.x)
    px = fma(-B, v.y, v.x);
    py = fma(B, v.x, v.y);
  } else {               // w v = A (B v.x - v.y, B v.y + v.x)
    px = fma(B, v.x, -v.y);
    py = fma(B, v.y, v.x);
  }
  const double2 a = u;
  u = make_double2(fma(A, px, a.x), fma(A, py, a.y));
  v = make_double2(fma(-A, px, a.x), fma(-A, py, a.y));
}

// Stage K (1..5) of the reduction tree of X^32 - exp(2 pi i TH0 / 128): node g splits
// X^(2h) - c into X^h - s and X^h + s, s = sqrt(c) = exp(2 pi i (TH0 + 128 br(g)) / 2^K / 128).
template <int K, int TH0, bool CB>
__device__ __forceinline__ void crt_stage(double2 (&x)[FFT_R]) {
  constexpr int H = 32 >> K;
#pragma unroll
  for (int g = 0; g < (1 << (K - 1)); ++g) {
    const int e = (TH0 + 128 * bitrev_bits(g, K - 1)) >> K;
#pragma unroll
    for (int j = 0; j < H; ++j) ct_bfly<CB>(e, x[2 * H * g + j], x[2 * H * g + j + H]);
  }
}

// Evaluation of sum_m x_m X^m at the roots of X^32 = exp(2 pi i TH0 / 128): register r ends up
// holding the value at exp(2 pi i (TH0 / 32 + 4 br(r)) / 128).
template <int TH0, bool CB>
__device__ __forceinline__ void crt_dft32(double2 (&x)[FFT_R]) {
  crt_stage<1, TH0, CB>(x);
  crt_stage<2, TH0, CB>(x);
  crt_stage<3, TH0, CB>(x);
  crt_stage<4, TH0, CB>(x);
  crt_stage<5, TH0, CB>(x);
}

// Butterfly of stage K (1..5) of the reduction tree of X^32 - exp(2 pi i TH0 / 128) on the pair
// (i, i + H), H = 32 >> K, as crt_stage<K, TH0> does it.
template <int K, int TH0, bool CB>
__device__ __forceinline__ void crt_bfly_at(double2 (&x)[FFT_R], int i) {
  constexpr int H = 32 >> K;
  const int e = (TH0 + 128 * bitrev_bits(i / (2 * H), K - 1)) >> K;
  ct_bfly<CB>(e, x[i], x[i + H]);
}

// crt_dft32<TH0> over inputs that `src(m)` produces (the value for register m), with every
// butterfly of stages 1-4 issued as soon as its operands exist: the input pairs (r, r + 16) come
// in 4-bit bit-reversed order of r, so after pairs r and r + 8 stage 2 can run on them, after four
// pairs stage 3, after eight stage 4.  The integer work that forms the inputs and the FP64
// butterflies then interleave in one instruction stream; every value meets the same butterflies
// in the same order as in crt_dft32, so the results are identical.
template <int TH0, bool CB, typename Src>
__device__ __forceinline__ void crt_dft32_from(double2 (&x)[FFT_R], Src&& src) {
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int r = bitrev_bits(k, 4);
    x[r] = src(r);
    x[r + 16] = src(r + 16);
    crt_bfly_at<1, TH0, CB>(x, r);
    if (k & 1) {  // pairs r - 8 and r are in
      crt_bfly_at<2, TH0, CB>(x, r - 8);
      crt_bfly_at<2, TH0, CB>(x, r + 8);
    }
    if ((k & 3) == 3) {  // every pair of residue j mod 4 is in
      const int j = bitrev_bits(k - 3, 4);
#pragma unroll
      for (int q = 0; q < 4; ++q) crt_bfly_at<3, TH0, CB>(x, 8 * q + j);
    }
    if ((k & 7) == 7) {  // every pair of residue j mod 2 is in
      const int j = bitrev_bits(k - 7, 4);
#pragma unroll
      for (int q = 0; q < 8; ++q) crt_bfly_at<4, TH0, CB>(x, 4 * q + j);
    }
  }
  crt_stage<5, TH0, CB>(x);
}

// Decimation-in-time stage of span 2^K: twiddle exp(-2 pi i j / 2^K) on the upper element.
template <int K, bool CB>
__device__ __forceinline__ void dit_stage(double2 (&x)[FFT_R]) {
  constexpr int LEN = 1 << K, HALF = LEN / 2;
#pragma unroll
  for (int s = 0; s < 32; s += LEN) {
#pragma unroll
    for (int j = 0; j < HALF; ++j) ct_bfly<CB>(128 - j * (128 >> K), x[s + j], x[s + j + HALF]);
  }
}

// Stages 1-3 of dit_dft32 on registers 8b..8b+7 alone (those stages never mix blocks of eight),
// so a block can be transformed as soon as its inputs exist; the butterflies are dit_stage's.
template <bool CB>
__device__ __forceinline__ void dit_block8(double2 (&x)[FFT_R], int b) {
  const int s0 = 8 * b;
#pragma unroll
  for (int s = 0; s < 8; s += 2) ct_bfly<CB>(128, x[s0 + s], x[s0 + s + 1]);
#pragma unroll
  for (int s = 0; s < 8; s += 4) {
#pragma unroll
    for (int j = 0; j < 2; ++j) ct_bfly<CB>(128 - 32 * j, x[s0 + s + j], x[s0 + s + j + 2]);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) ct_bfly<CB>(128 - 16 * j, x[s0 + j], x[s0 + j + 4]);
}

// out_k = sum_n in_n exp(-2 pi i n k / 32) with in_n in register br(n), out_k in register k.
template <bool CB>
__device__ __forceinline__ void dit_dft32(double2 (&x)[FFT_R]) {
  dit_stage<1, CB>(x);
  dit_stage<2, CB>(x);
  dit_stage<3, CB>(x);
  dit_stage<4, CB>(x);
  dit_stage<5, CB>(x);
}

// x_m *= exp(-2 pi i m / 128) * 2^-SHIFT, SHIFT = 10 (the 1/M), 26 or 42 (also the 2^-16 or
// 2^-32 a blind rotation's rounding expects); the constants come pre-scaled.
template <int SHIFT, bool CB>
__device__ __forceinline__ void untwist_at(double2 (&x)[FFT_R], int m) {
  static_assert(SHIFT == 10 || SHIFT == 26 || SHIFT == 42, "no untwist table for this scale");
  const double2* k = SHIFT == 10 ? kUntwist10 : SHIFT == 26 ? kUntwist26 : kUntwist42;
  constexpr double sc = 1.0 / (double)(1ull << SHIFT);
  double c, sn;
  if (CB) {
    c = k[m].x;
    sn = k[m].y;
  } else {
    cs128_lit((128 - m) & 127, c, sn);
    c *= sc;  // literals: folded at compile time
    sn *= sc;
  }
  x[m] = m == 0 ? make_double2(x[m].x * c, x[m].y * c) : cmul(x[m], make_double2(c, sn));
}

template <int SHIFT, bool CB>
__device__ __forceinline__ void untwist(double2 (&x)[FFT_R]) {
#pragma unroll
  for (int m = 0; m < 32; ++m) untwist_at<SHIFT, CB>(x, m);
}

// dit_dft32 followed by untwist<SHIFT>, handing every finished register m to `sink(m)` as soon
// as its last butterfly and its untwist are done: after stages 1-3, stages 4 and 5 run in eight
// chunks (stage-4 pairs (j, j + 8) and (16 + j, 24 + j), then stage-5 pairs (j, j + 16) and
// (j + 8, j + 24)), so the consumer's work on one chunk interleaves with the next chunk's
// butterflies.  The arithmetic per value is that of dit_dft32 and untwist, in the same order.
template <int SHIFT, bool CB, typename Sink>
__device__ __forceinline__ void dit_dft32_untwist_to(double2 (&x)[FFT_R], Sink&& sink) {
  dit_stage<1, CB>(x);
  dit_stage<2, CB>(x);
  dit_stage<3, CB>(x);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ct_bfly<CB>(128 - 8 * j, x[j], x[j + 8]);
    ct_bfly<CB>(128 - 8 * j, x[16 + j], x[24 + j]);
    ct_bfly<CB>(128 - 4 * j, x[j], x[j + 16]);
    ct_bfly<CB>(128 - 4 * (j + 8), x[j + 8], x[j + 24]);
    untwist_at<SHIFT, CB>(x, j);
    sink(j);
    untwist_at<SHIFT, CB>(x, j + 16);
    sink(j + 16);
    untwist_at<SHIFT, CB>(x, j + 8);
    sink(j + 8);
    untwist_at<SHIFT, CB>(x, j + 24);
    sink(j + 24);
  }
}

// Swizzled 32x32 transpose through a per-warp shared buffer of 1024 double2.
// Writes element (row = register index, col = lane) to slot row * 32 + (col ^ row) and reads
// back (row = lane, col = register): both patterns touch 32 distinct columns of distinct rows,
// so neither has bank conflicts, and each address is one XOR on a per-lane base.
__device__ __forceinline__ void warp_transpose(double2 (&x)[FFT_R], double2* buf, int lane) {
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + (lane ^ r)] = x[r];
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q] = buf[lane * 32 + (q ^ lane)];
  __syncwarp();
}

// The same transpose through an 8 KB buffer of 1024 doubles: real parts, then imaginary parts.
__device__ __forceinline__ void warp_transpose_half(double2 (&x)[FFT_R], double* buf, int lane) {
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + (lane ^ r)] = x[r].x;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q].x = buf[lane * 32 + (q ^ lane)];
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + (lane ^ r)] = x[r].y;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q].y = buf[lane * 32 + (q ^ lane)];
  __syncwarp();
}

// Read-only load the compiler may not hoist out of the blind-rotation loop: the twiddles are
// loop-invariant, and keeping all of them in registers across iterations would spill.
__device__ __forceinline__ double2 ld_tw(const double2* p) {
  double2 v;
  asm volatile("ld.global.nc.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "l"(p));
  return v;
}

// Forward transform with the twiddles T from global memory (through L1) and a 16 KB buffer.
template <bool CB = true>
__device__ __forceinline__ void fft_forward(double2 (&x)[FFT_R], double2* buf, int lane,
                                            const FftTables& tb) {
  crt_dft32<32, CB>(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], ld_tw(&tb.wf[r * 32 + lane]));
  warp_transpose(x, buf, lane);
  crt_dft32<0, CB>(x);
}

// Inverse transform back to folded coefficients scaled by 1/M.
template <bool CB = true>
__device__ __forceinline__ void fft_inverse(double2 (&x)[FFT_R], double2* buf, int lane,
                                            const FftTables& tb) {
  dit_dft32<CB>(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], ld_tw(&tb.wi[n * 32 + lane]));
  warp_transpose(x, buf, lane);
  dit_dft32<CB>(x);
  untwist<10, CB>(x);
}

// The same pair through the 8 KB half buffer, the twiddles read from global memory.
template <bool CB = true>
__device__ __forceinline__ void fft_forward_h(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_g) {
  crt_dft32<32, CB>(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], __ldg(&wf_g[r * 32 + lane]));
  warp_transpose_half(x, buf, lane);
  crt_dft32<0, CB>(x);
}

template <bool CB = true, int SHIFT = 10>
__device__ __forceinline__ void fft_inverse_h(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wi_g) {
  dit_dft32<CB>(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], __ldg(&wi_g[n * 32 + lane]));
  warp_transpose_half(x, buf, lane);
  dit_dft32<CB>(x);
  untwist<SHIFT, CB>(x);
}

// Twiddle table T held once in shared memory for both directions.  Element (a, b) of the 32x32
// table lives at a*32 + (a ^ b): the forward transform reads row r across the lanes and the
// inverse reads the transpose (its twiddle at lane l, register n is conj(T(l, n))); with this
// swizzle both patterns are bank-conflict free.
__device__ __forceinline__ int tw_swz(int a, int b) { return a * 32 + (a ^ b); }

template <bool CB = true>
__device__ __forceinline__ void fft_forward_s(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_sw) {
  crt_dft32<32, CB>(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], wf_sw[tw_swz(r, lane)]);
  warp_transpose_half(x, buf, lane);
  crt_dft32<0, CB>(x);
}

// Inverse scaled by 2^-SHIFT overall (SHIFT >= 10 includes the 1/M).
template <int SHIFT, bool CB = true>
__device__ __forceinline__ void fft_inverse_s(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_sw) {
  dit_dft32<CB>(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul_conj(x[n], wf_sw[tw_swz(lane, n)]);
  warp_transpose_half(x, buf, lane);
  dit_dft32<CB>(x);
  untwist<SHIFT, CB>(x);
}

// Host: build (once per device) and fetch the tables of the current device.
int fft_tables_get(FftTables* out);

}  // namespace pnb
